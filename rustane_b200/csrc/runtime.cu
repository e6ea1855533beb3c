// Model-level C ABI of librustane_cuda: context, device arenas, host<->device
// transfers and the orchestration of forward, backward and AdamW.
//
// The orchestration restates the reference engine in token-major form:
//   full_model::forward_ws  (crates/engine/src/full_model.rs:187-247)
//   layer::forward_into     (crates/engine/src/layer.rs:552-680)
//   full_model::backward_ws (full_model.rs:250-331)
//   layer::backward_into    (layer.rs:1606-1858)
//   full_model::update_weights / grad_norm / train_step (full_model.rs:490-714)
// Every heavy step runs in one of the sm_100a kernels (gemm.cu, attention.cu,
// elementwise.cu); there is no CPU compute path.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <mutex>
#include <set>
#include <thread>
#include <utility>

#include "attention.h"
#include "common.cuh"
#include "elementwise.h"
#include "kernels.h"
#include "runtime.h"

using rt::bf16;

// ============================================ per-device kernel attributes
namespace rt {
cudaError_t smem_limit_once(const void* fn, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;  // (kernel, device)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({fn, dev})) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert({fn, dev});
  return e;
}
}  // namespace rt

// ================================================================ NCCL (dlopen)
namespace rt {
struct NcclApi {
  void* handle = nullptr;
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRank) commInitRank = nullptr;
  decltype(&ncclAllReduce) allReduce = nullptr;
  decltype(&ncclReduceScatter) reduceScatter = nullptr;
  decltype(&ncclAllGather) allGather = nullptr;
  decltype(&ncclGroupStart) groupStart = nullptr;
  decltype(&ncclGroupEnd) groupEnd = nullptr;
  decltype(&ncclCommGetAsyncError) getAsyncError = nullptr;
  decltype(&ncclCommCount) commCount = nullptr;
  decltype(&ncclCommAbort) commAbort = nullptr;
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclGetErrorString) errorString = nullptr;
};
struct NcclState {
  ncclComm_t comm = nullptr;
  bool aborted = false;
};

static NcclApi* nccl_api() {
  static NcclApi api;
  static bool tried = false;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (tried) return api.handle ? &api : nullptr;
  tried = true;
  const char* env = getenv("RUSTANE_NCCL_LIB");
  void* h = nullptr;
  if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);  // already loaded (e.g. by torch)
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return nullptr;
  api.handle = h;
#define RT_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
  RT_SYM(getUniqueId, "ncclGetUniqueId");
  RT_SYM(commInitRank, "ncclCommInitRank");
  RT_SYM(allReduce, "ncclAllReduce");
  RT_SYM(reduceScatter, "ncclReduceScatter");
  RT_SYM(allGather, "ncclAllGather");
  RT_SYM(groupStart, "ncclGroupStart");
  RT_SYM(groupEnd, "ncclGroupEnd");
  RT_SYM(getAsyncError, "ncclCommGetAsyncError");
  RT_SYM(commCount, "ncclCommCount");
  RT_SYM(commAbort, "ncclCommAbort");
  RT_SYM(commDestroy, "ncclCommDestroy");
  RT_SYM(errorString, "ncclGetErrorString");
#undef RT_SYM
  if (!api.getUniqueId || !api.commInitRank || !api.allReduce || !api.getAsyncError || !api.commAbort ||
      !api.commDestroy) {
    api.handle = nullptr;
    return nullptr;
  }
  return &api;
}
}  // namespace rt

// ================================================================ helpers
namespace {

int set_err(rt_ctx* c, int code, const std::string& msg) {
  if (c) c->last_error = msg;
  return code;
}

int cuda_err(rt_ctx* c, cudaError_t e, const char* what) {
  return set_err(c, RT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define RT_CUDA(call, what)                        \
  do {                                             \
    cudaError_t _e = (call);                       \
    if (_e != cudaSuccess) return cuda_err(c, _e, what); \
  } while (0)

#define RT_LAUNCH(call, what)                                                                     \
  do {                                                                                            \
    int _rc = (call);                                                                             \
    if (_rc != 0)                                                                                 \
      return set_err(c, _rc == -1 ? RT_ERR_SHAPE : RT_ERR_CUDA,                                   \
                     std::string(what) + " launch failed (" + std::to_string(_rc) + ")");         \
  } while (0)

template <class T>
T* dalloc(rt_ctx* c, int64_t count) {
  if (count <= 0) return nullptr;
  size_t bytes = (static_cast<size_t>(count) * sizeof(T) + 255) & ~size_t(255);
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
  c->allocations.push_back({p, bytes});
  c->device_bytes += static_cast<int64_t>(bytes);
  return static_cast<T*>(p);
}

void dfree(rt_ctx* c, void* p) {
  if (!p) return;
  for (size_t i = 0; i < c->allocations.size(); ++i)
    if (c->allocations[i].first == p) {
      c->device_bytes -= static_cast<int64_t>(c->allocations[i].second);
      c->allocations.erase(c->allocations.begin() + static_cast<long>(i));
      cudaFree(p);
      return;
    }
}

cudaEvent_t pool_event(rt_ctx* c) {
  if (c->event_pool_used == c->event_pool.size()) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    c->event_pool.push_back(e);
  }
  return c->event_pool[c->event_pool_used++];
}

// Run one launcher, count its kernels and time it when profiling.
template <class F>
int launch_on(rt_ctx* c, cudaStream_t st, int kind, double flops, int nkernels, F&& f) {
  cudaEvent_t a = nullptr, b = nullptr;
  if (c->profiling) {
    a = pool_event(c);
    cudaEventRecord(a, st);
  }
  const int rc = f();
  if (c->profiling) {
    b = pool_event(c);
    cudaEventRecord(b, st);
    c->kevents.push_back({kind, flops, a, b});
  }
  c->acc.kernel_launches += nkernels;
  if (kind == 0) c->acc.gemm_launches += nkernels;
  else if (kind == 1) c->acc.attn_launches += nkernels;
  else c->acc.other_launches += nkernels;
  return rc;
}
template <class F>
int launch(rt_ctx* c, int kind, double flops, int nkernels, F&& f) {
  return launch_on(c, c->stream, kind, flops, nkernels, f);
}

void harvest_kernel_events(rt_ctx* c) {
  for (const auto& k : c->kevents) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, k.a, k.b) != cudaSuccess) continue;
    if (k.kind == 0) {
      c->acc.gemm_ms += ms;
      c->acc.gemm_flops += k.flops;
    } else if (k.kind == 1) {
      c->acc.attn_ms += ms;
      c->acc.attn_flops += k.flops;
    } else {
      c->acc.other_ms += ms;
    }
  }
  c->kevents.clear();
  c->event_pool_used = 0;
}

int gemm(rt_ctx* c, rt::GemmArgs g, const char* what, cudaStream_t st = nullptr) {
  g.err = c->d_err;
  if (!st) st = c->stream;
  const double n_out = g.epi == rt::kEpiSwiglu ? 2.0 * g.N : double(g.N);
  const double fl = 2.0 * double(g.M) * n_out * double(g.K);
  RT_LAUNCH(launch_on(c, st, 0, fl, 1, [&] { return rt::gemm_launch(g, st); }), what);
  return RT_OK;
}

int other(rt_ctx* c, int nk, int rc_in, const char* what) {
  (void)nk;
  if (rc_in != 0)
    return set_err(c, rc_in == -1 ? RT_ERR_SHAPE : RT_ERR_CUDA,
                   std::string(what) + " launch failed (" + std::to_string(rc_in) + ")");
  return RT_OK;
}

#define RT_OTHER(nk, expr, what) \
  do {                           \
    int _r = launch(c, 2, 0.0, nk, [&] { return (expr); }); \
    if (_r != 0) return other(c, nk, _r, what); \
  } while (0)
#define RT_OTHER_ON(st, nk, expr, what) \
  do {                                  \
    int _r = launch_on(c, st, 2, 0.0, nk, [&] { return (expr); }); \
    if (_r != 0) return other(c, nk, _r, what); \
  } while (0)

bool forward_only(const rt_ctx* c) { return (c->flags & RT_CTX_FORWARD_ONLY) != 0; }
float alpha_of(const rt_model_config& cfg) { return 1.0f / std::sqrt(2.0f * static_cast<float>(cfg.nlayers)); }

// Gamma pointers: training arenas keep them after the matrices; forward-only
// contexts keep [embed | gammas] in a compact fp32 buffer.
float* gamma_base(rt_ctx* c) { return c->params + (forward_only(c) ? c->n_embed : c->n_matrix_end); }

// The main stream waits for the weight all-gathers a sharded train step left on
// the comm stream (asynchronous; the next forward waits for them layer by layer
// instead).
void join_gathers(rt_ctx* c) {
  if (c->gather_pending) {
    cudaStreamWaitEvent(c->stream, c->ev_gather_all, 0);
    c->gather_pending = false;
  }
}

// Wait for the stream; with a communicator, poll so that a stuck collective
// aborts after timeout_ms instead of blocking forever.
int wait_stream(rt_ctx* c) {
  join_gathers(c);
  if (!c->nccl || !c->nccl->comm) {
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return cuda_err(c, e, "stream synchronize");
  } else {
    rt::NcclApi* api = rt::nccl_api();
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
      cudaError_t q = cudaStreamQuery(c->stream);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return cuda_err(c, q, "stream query");
      ncclResult_t ar = ncclSuccess;
      api->getAsyncError(c->nccl->comm, &ar);
      const auto ms =
          std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
      if ((ar != ncclSuccess && ar != ncclInProgress) || (c->timeout_ms > 0 && ms > c->timeout_ms)) {
        api->commAbort(c->nccl->comm);
        c->nccl->comm = nullptr;
        c->nccl->aborted = true;
        return set_err(c, RT_ERR_NCCL, ar != ncclSuccess ? std::string("NCCL async error: ") + api->errorString(ar)
                                                         : "NCCL collective timed out; communicator aborted");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
  int herr = 0;
  cudaError_t e = cudaMemcpy(&herr, c->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_err(c, e, "read device error word");
  if (herr != 0) {
    cudaMemset(c->d_err, 0, sizeof(int));
    return set_err(c, herr == rt::kDevBadToken ? RT_ERR_TOKEN : RT_ERR_DEVICE,
                   "device error code " + std::to_string(herr) +
                       (herr <= 3 ? " (pipeline wait timed out)" : herr == 4 ? " (token id out of range)" : ""));
  }
  if (c->profiling) harvest_kernel_events(c);
  return RT_OK;
}

void compute_rope_tables(const rt_model_config& cfg, std::vector<float>& cf, std::vector<float>& sf,
                         std::vector<float>& cb, std::vector<float>& sb) {
  const int S = cfg.seq, hd = cfg.hd, pairs = hd / 2;
  cf.assign(size_t(S) * pairs, 0.f);
  sf.assign(size_t(S) * pairs, 0.f);
  cb.assign(size_t(pairs) * S, 0.f);
  sb.assign(size_t(pairs) * S, 0.f);
  for (int p = 0; p < S; ++p)
    for (int i = 0; i < pairs; ++i) {  // kernels/sdpa_fwd.rs:18-33
      const float theta = static_cast<float>(p) / powf(10000.0f, 2.0f * static_cast<float>(i) / static_cast<float>(hd));
      cf[size_t(p) * pairs + i] = cosf(theta);
      sf[size_t(p) * pairs + i] = sinf(theta);
    }
  for (int i = 0; i < pairs; ++i) {  // layer.rs:203-216
    const float freq = 1.0f / powf(10000.0f, 2.0f * static_cast<float>(i) / static_cast<float>(hd));
    for (int p = 0; p < S; ++p) {
      const float theta = static_cast<float>(p) * freq;
      cb[size_t(i) * S + p] = cosf(theta);
      sb[size_t(i) * S + p] = sinf(theta);
    }
  }
}

// ------------------------------------------------------------ host copies
// Copy a [rows, cols] host matrix into columns [col0, col0+cols) of a device
// matrix with row stride ld (elements), or back.  Every host <-> device copy of
// the context is ordered on its own (non-blocking) stream: a plain cudaMemcpy
// from pageable memory may return before its DMA lands and is not ordered with
// kernels on a non-blocking stream.
int copy_block_h2d(rt_ctx* c, float* dst, int64_t ld, int64_t col0, const float* src, int64_t rows, int64_t cols,
                   int64_t src_ld = 0) {
  if (src_ld == 0) src_ld = cols;
  RT_CUDA(cudaMemcpy2DAsync(dst + col0, ld * sizeof(float), src, src_ld * sizeof(float), cols * sizeof(float), rows,
                       cudaMemcpyHostToDevice, c->stream),
          "upload");
  return RT_OK;
}
int copy_block_d2h(rt_ctx* c, float* dst, const float* src, int64_t ld, int64_t col0, int64_t rows, int64_t cols) {
  RT_CUDA(cudaMemcpy2DAsync(dst, cols * sizeof(float), src + col0, ld * sizeof(float), cols * sizeof(float), rows,
                       cudaMemcpyDeviceToHost, c->stream),
          "download");
  return RT_OK;
}

// Host tensors <-> one fp32 arena laid out like the parameters.
int arena_h2d(rt_ctx* c, float* arena, const rt_model_ptrs* h) {
  const auto& cfg = c->cfg;
  const int64_t D = cfg.dim, H = cfg.hidden, Q = cfg.q_dim;
  if (!h || !h->embed || !h->gamma_final || !h->layers) return set_err(c, RT_ERR_ARG, "null model pointers");
  RT_CUDA(cudaMemcpyAsync(arena, h->embed, sizeof(float) * cfg.vocab * D, cudaMemcpyHostToDevice, c->stream), "upload embed");
  float* gb = arena + c->n_matrix_end;
  RT_CUDA(cudaMemcpyAsync(gb, h->gamma_final, sizeof(float) * D, cudaMemcpyHostToDevice, c->stream), "upload gamma_final");
  for (int l = 0; l < cfg.nlayers; ++l) {
    const rt_layer_ptrs& L = h->layers[l];
    const auto& o = c->layer_off[l];
    if (!L.wq || !L.wk || !L.wv || !L.wo || !L.w1 || !L.w3 || !L.w2 || !L.gamma1 || !L.gamma2)
      return set_err(c, RT_ERR_ARG, "null layer pointer");
    int rc;
    if ((rc = copy_block_h2d(c, arena + o.wqkv, 3 * D, 0, L.wq, D, D))) return rc;
    if ((rc = copy_block_h2d(c, arena + o.wqkv, 3 * D, D, L.wk, D, D))) return rc;
    if ((rc = copy_block_h2d(c, arena + o.wqkv, 3 * D, 2 * D, L.wv, D, D))) return rc;
    RT_CUDA(cudaMemcpyAsync(arena + o.wo, L.wo, sizeof(float) * Q * D, cudaMemcpyHostToDevice, c->stream), "upload wo");
    if ((rc = copy_block_h2d(c, arena + o.w13, 2 * H, 0, L.w1, D, H))) return rc;
    if ((rc = copy_block_h2d(c, arena + o.w13, 2 * H, H, L.w3, D, H))) return rc;
    RT_CUDA(cudaMemcpyAsync(arena + o.w2, L.w2, sizeof(float) * D * H, cudaMemcpyHostToDevice, c->stream), "upload w2");
    RT_CUDA(cudaMemcpyAsync(arena + o.gamma1, L.gamma1, sizeof(float) * D, cudaMemcpyHostToDevice, c->stream), "upload gamma1");
    RT_CUDA(cudaMemcpyAsync(arena + o.gamma2, L.gamma2, sizeof(float) * D, cudaMemcpyHostToDevice, c->stream), "upload gamma2");
  }
  return RT_OK;
}

int arena_d2h(rt_ctx* c, const float* arena, const rt_model_ptrs* h) {
  const auto& cfg = c->cfg;
  const int64_t D = cfg.dim, H = cfg.hidden, Q = cfg.q_dim;
  if (!h || !h->embed || !h->gamma_final || !h->layers) return set_err(c, RT_ERR_ARG, "null model pointers");
  RT_CUDA(cudaMemcpyAsync(h->embed, arena, sizeof(float) * cfg.vocab * D, cudaMemcpyDeviceToHost, c->stream), "download embed");
  RT_CUDA(cudaMemcpyAsync(h->gamma_final, arena + c->n_matrix_end, sizeof(float) * D, cudaMemcpyDeviceToHost, c->stream),
          "download gamma_final");
  for (int l = 0; l < cfg.nlayers; ++l) {
    const rt_layer_ptrs& L = h->layers[l];
    const auto& o = c->layer_off[l];
    int rc;
    if ((rc = copy_block_d2h(c, L.wq, arena + o.wqkv, 3 * D, 0, D, D))) return rc;
    if ((rc = copy_block_d2h(c, L.wk, arena + o.wqkv, 3 * D, D, D, D))) return rc;
    if ((rc = copy_block_d2h(c, L.wv, arena + o.wqkv, 3 * D, 2 * D, D, D))) return rc;
    RT_CUDA(cudaMemcpyAsync(L.wo, arena + o.wo, sizeof(float) * Q * D, cudaMemcpyDeviceToHost, c->stream), "download wo");
    if ((rc = copy_block_d2h(c, L.w1, arena + o.w13, 2 * H, 0, D, H))) return rc;
    if ((rc = copy_block_d2h(c, L.w3, arena + o.w13, 2 * H, H, D, H))) return rc;
    RT_CUDA(cudaMemcpyAsync(L.w2, arena + o.w2, sizeof(float) * D * H, cudaMemcpyDeviceToHost, c->stream), "download w2");
    RT_CUDA(cudaMemcpyAsync(L.gamma1, arena + o.gamma1, sizeof(float) * D, cudaMemcpyDeviceToHost, c->stream), "download gamma1");
    RT_CUDA(cudaMemcpyAsync(L.gamma2, arena + o.gamma2, sizeof(float) * D, cudaMemcpyDeviceToHost, c->stream), "download gamma2");
  }
  return RT_OK;
}

int materialize_zero_grads(rt_ctx* c) {
  if (c->grads_zero_pending) {
    RT_CUDA(cudaMemsetAsync(c->grads, 0, sizeof(float) * c->n_params, c->stream), "zero grads");
    c->grads_zero_pending = false;
    c->sharded_g = false;
  }
  return RT_OK;
}

void alloc_token_batch(rt_ctx* c, rt::TokenBatch& tb) {
  const int64_t M = int64_t(c->max_batch) * c->cfg.seq;
  tb.tokens = dalloc<uint32_t>(c, M);
  tb.targets = dalloc<uint32_t>(c, M);
  tb.perm = dalloc<int32_t>(c, M);
  tb.seg_start = dalloc<int32_t>(c, M + 1);
  tb.seg_tok = dalloc<uint32_t>(c, M);
}

// Tokens -> device, with the embedding-scatter segments built on the host
// (counting sort by token, positions ascending within a token).
int upload_tokens(rt_ctx* c, rt::TokenBatch& tb, const uint32_t* tokens, const uint32_t* targets, int batch) {
  const int M = batch * c->cfg.seq;
  const uint32_t V = static_cast<uint32_t>(c->cfg.vocab);
  for (int i = 0; i < M; ++i)
    if (tokens[i] >= V || (targets && targets[i] >= V))
      return set_err(c, RT_ERR_TOKEN, "token id " + std::to_string(tokens[i] >= V ? tokens[i] : targets[i]) +
                                          " at position " + std::to_string(i) + " >= vocab " + std::to_string(V));
  uint32_t* st_tok = static_cast<uint32_t*>(c->h_stage);
  uint32_t* st_tgt = st_tok + M;
  int32_t* st_perm = reinterpret_cast<int32_t*>(st_tgt + M);
  int32_t* st_start = st_perm + M;
  uint32_t* st_segtok = reinterpret_cast<uint32_t*>(st_start + M + 1);
  memcpy(st_tok, tokens, sizeof(uint32_t) * M);
  if (targets) memcpy(st_tgt, targets, sizeof(uint32_t) * M);
  std::vector<int32_t> count(V + 1, 0);
  for (int i = 0; i < M; ++i) count[tokens[i] + 1]++;
  for (uint32_t v = 0; v < V; ++v) count[v + 1] += count[v];
  int nseg = 0;
  for (uint32_t v = 0; v < V; ++v)
    if (count[v + 1] > count[v]) {
      st_start[nseg] = count[v];
      st_segtok[nseg] = v;
      ++nseg;
    }
  st_start[nseg] = M;
  std::vector<int32_t> fillpos(count.begin(), count.end() - 1);
  for (int i = 0; i < M; ++i) st_perm[fillpos[tokens[i]]++] = i;
  tb.nseg = nseg;
  tb.batch = batch;
  RT_CUDA(cudaMemcpyAsync(tb.tokens, st_tok, sizeof(uint32_t) * M, cudaMemcpyHostToDevice, c->stream), "tokens");
  if (targets)
    RT_CUDA(cudaMemcpyAsync(tb.targets, st_tgt, sizeof(uint32_t) * M, cudaMemcpyHostToDevice, c->stream),
            "targets");
  RT_CUDA(cudaMemcpyAsync(tb.perm, st_perm, sizeof(int32_t) * M, cudaMemcpyHostToDevice, c->stream), "perm");
  RT_CUDA(cudaMemcpyAsync(tb.seg_start, st_start, sizeof(int32_t) * (nseg + 1), cudaMemcpyHostToDevice, c->stream),
          "seg_start");
  RT_CUDA(cudaMemcpyAsync(tb.seg_tok, st_segtok, sizeof(uint32_t) * nseg, cudaMemcpyHostToDevice, c->stream),
          "seg_tok");
  c->h2d_bytes_last = int64_t(sizeof(uint32_t)) * (targets ? 2 * M : M) + int64_t(sizeof(int32_t)) * (M + nseg + 1) +
                      int64_t(sizeof(uint32_t)) * nseg;
  return RT_OK;
}

// bf16 weight arena: [embed | per layer Wqkv D x 3Dl, Wo Dl x D, W13 D x 2Hl, W2 D x Hl] with
// Dl = this rank's heads * hd and Hl its hidden columns (the full sizes without TP).
void layout_bf16(rt_ctx* c) {
  const int64_t D = c->cfg.dim, Dl = int64_t(c->heads_loc) * c->cfg.hd, Hl = c->hid_loc;
  c->layer_off_b.resize(c->cfg.nlayers);
  int64_t off = int64_t(c->cfg.vocab) * D;
  for (auto& o : c->layer_off_b) {
    o.wqkv = off;
    off += D * 3 * Dl;
    o.wo = off;
    off += Dl * D;
    o.w13 = off;
    off += D * 2 * Hl;
    o.w2 = off;
    off += D * Hl;
    o.gamma1 = o.gamma2 = 0;
  }
  c->n_bf16 = off;
}

// Buffers whose size depends on the shard: bf16 weights, q/k/v, attention
// output, lse, h1|h3, gate, and the TP partial.  Returns false on OOM.
bool alloc_shard_buffers(rt_ctx* c) {
  const int64_t M = int64_t(c->max_batch) * c->cfg.seq, Dl = int64_t(c->heads_loc) * c->cfg.hd, Hl = c->hid_loc;
  bool ok = true;
  auto need = [&](void* p) { ok = ok && p != nullptr; };
  c->params_bf16 = dalloc<bf16>(c, c->n_bf16);
  need(c->params_bf16);
  for (auto& A : c->acts) {
    A.qkv = dalloc<bf16>(c, M * 3 * Dl);
    A.attn = dalloc<bf16>(c, M * Dl);
    A.lse2 = dalloc<float>(c, M * c->heads_loc);
    A.h13 = dalloc<bf16>(c, M * 2 * Hl);
    A.gate = dalloc<bf16>(c, M * Hl);
    for (void* p : {(void*)A.qkv, (void*)A.attn, (void*)A.lse2, (void*)A.h13, (void*)A.gate}) need(p);
  }
  if (c->tp) {
    c->tp_partial = dalloc<bf16>(c, M * c->cfg.dim);
    need(c->tp_partial);
  }
  return ok;
}

void free_shard_buffers(rt_ctx* c) {
  dfree(c, c->params_bf16);
  c->params_bf16 = nullptr;
  for (auto& A : c->acts) {
    for (void* p : {(void*)A.qkv, (void*)A.attn, (void*)A.lse2, (void*)A.h13, (void*)A.gate}) dfree(c, p);
    A.qkv = A.attn = A.h13 = A.gate = nullptr;
    A.lse2 = nullptr;
  }
  dfree(c, c->tp_partial);
  c->tp_partial = nullptr;
}

// Sum of the row-parallel GEMM partials over the tensor-parallel ranks (bf16).
int tp_allreduce(rt_ctx* c, int64_t n) {
  rt::NcclApi* api = rt::nccl_api();
  if (!api || !c->nccl || !c->nccl->comm) return set_err(c, RT_ERR_NCCL, "no communicator (aborted or not initialised)");
  ncclResult_t r = api->allReduce(c->tp_partial, c->tp_partial, static_cast<size_t>(n), ncclBfloat16, ncclSum,
                                  c->nccl->comm, c->stream);
  if (r != ncclSuccess) return set_err(c, RT_ERR_NCCL, std::string("ncclAllReduce: ") + api->errorString(r));
  return RT_OK;
}

// ---------------------------------------------------------------- forward
int layer_forward(rt_ctx* c, int l, const rt::LayerActs& A, const float* x_in, float* x_next, int batch) {
  const auto& cfg = c->cfg;
  const int D = cfg.dim, S = cfg.seq, M = batch * S;
  const int Dl = c->heads_loc * cfg.hd, Hl = c->hid_loc;  // this rank's shard (everything without TP)
  const float alpha = alpha_of(cfg);
  const auto& o = c->layer_off[l];
  const auto& ob = c->layer_off_b[l];
  const bf16* W = c->params_bf16;
  const float* G = gamma_base(c);
  const int64_t goff = c->n_matrix_end;  // gamma offsets are relative to gamma_base()
  int rc;
  RT_OTHER(1, rt::rmsnorm_fwd(x_in, G + (o.gamma1 - goff), A.xn, A.rms1, M, D, c->stream), "rmsnorm1");
  {  // Q K V projection + RoPE (sdpaFwd, kernels/sdpa_fwd.rs:80-128); TP: this rank's heads
    rt::GemmArgs g;
    g.a = A.xn; g.lda = D;
    g.b = W + ob.wqkv; g.ldb = 3 * Dl; g.b_mn = true;
    g.M = M; g.N = 3 * Dl; g.K = D;
    g.epi = rt::kEpiRope; g.out = A.qkv; g.ldo = 3 * Dl;
    g.rope_cos = c->rope_cos_f; g.rope_sin = c->rope_sin_f; g.seq = S; g.rope_cols = 2 * Dl;
    if ((rc = gemm(c, g, "qkv"))) return rc;
  }
  {  // causal attention (sdpa_fwd.rs:130-150)
    rt::AttnArgs a;
    a.batch = batch; a.S = S; a.heads = c->heads_loc; a.hd = cfg.hd; a.D = Dl;
    a.qkv = A.qkv; a.ldq = 3 * Dl; a.out = A.attn; a.ldo = Dl; a.lse2 = A.lse2; a.err = c->d_err;
    const double fl = 4.0 * batch * c->heads_loc * double(S) * S / 2.0 * cfg.hd;
    RT_LAUNCH(launch(c, 1, fl, 1, [&] { return rt::attn_forward(a, c->stream); }), "attention fwd");
  }
  if (!c->tp) {  // woFwd + residual x2 = x + alpha * o (layer.rs:769-784)
    rt::GemmArgs g;
    g.a = A.attn; g.lda = Dl;
    g.b = W + ob.wo; g.ldb = D; g.b_mn = true;
    g.M = M; g.N = D; g.K = Dl;
    g.epi = rt::kEpiResidual; g.aux = x_in; g.ld_aux = D; g.out = A.x2; g.ldo = D; g.alpha = alpha;
    if ((rc = gemm(c, g, "wo"))) return rc;
    RT_OTHER(1, rt::rmsnorm_fwd(A.x2, G + (o.gamma2 - goff), A.x2n, A.rms2, M, D, c->stream), "rmsnorm2");
  } else {  // row-parallel Wo: partial -> all-reduce -> x2 = x + alpha * sum, RMSNorm2
    rt::GemmArgs g;
    g.a = A.attn; g.lda = Dl;
    g.b = W + ob.wo; g.ldb = D; g.b_mn = true;
    g.M = M; g.N = D; g.K = Dl;
    g.epi = rt::kEpiBf16; g.out = c->tp_partial; g.ldo = D;
    if ((rc = gemm(c, g, "wo (row-parallel)"))) return rc;
    if ((rc = tp_allreduce(c, int64_t(M) * D))) return rc;
    RT_OTHER(1, rt::residual_rmsnorm_fwd(x_in, c->tp_partial, alpha, G + (o.gamma2 - goff), A.x2, A.x2n, A.rms2, M,
                                         D, c->stream),
             "residual + rmsnorm2");
  }
  {  // W1 | W3 + SwiGLU (ffn_fused.rs:46-63); TP: this rank's hidden columns
    rt::GemmArgs g;
    g.a = A.x2n; g.lda = D;
    g.b = W + ob.w13; g.ldb = 2 * Hl; g.b_mn = true;
    g.M = M; g.N = Hl; g.K = D;
    g.epi = rt::kEpiSwiglu; g.out = A.h13; g.ldo = 2 * Hl; g.out2 = A.gate; g.ldo2 = Hl; g.n_half = Hl;
    if ((rc = gemm(c, g, "w13"))) return rc;
  }
  {  // gate W2^T + residual (ffn_fused.rs:65-78); TP: row-parallel + all-reduce
    rt::GemmArgs g;
    g.a = A.gate; g.lda = Hl;
    g.b = W + ob.w2; g.ldb = Hl; g.b_mn = false;
    g.M = M; g.N = D; g.K = Hl;
    if (!c->tp) {
      g.epi = rt::kEpiResidual; g.aux = A.x2; g.ld_aux = D; g.out = x_next; g.ldo = D; g.alpha = alpha;
      if ((rc = gemm(c, g, "w2"))) return rc;
    } else {
      g.epi = rt::kEpiBf16; g.out = c->tp_partial; g.ldo = D;
      if ((rc = gemm(c, g, "w2 (row-parallel)"))) return rc;
      if ((rc = tp_allreduce(c, int64_t(M) * D))) return rc;
      RT_OTHER(1, rt::residual_rmsnorm_fwd(A.x2, c->tp_partial, alpha, nullptr, x_next, nullptr, nullptr, M, D,
                                           c->stream),
               "residual");
    }
  }
  return RT_OK;
}

int forward_impl(rt_ctx* c, int batch, float softcap) {
  const auto& cfg = c->cfg;
  const int D = cfg.dim, V = cfg.vocab, M = batch * cfg.seq;
  int rc;
  cudaEventRecord(c->ev[0], c->stream);
  const bool pend = c->gather_pending;  // weights of the last sharded step still arriving, segment by segment
  if (pend) {
    cudaStreamWaitEvent(c->stream, c->ev_gather_seg.back(), 0);  // gammas
    cudaStreamWaitEvent(c->stream, c->ev_gather_seg[0], 0);      // embedding (fp32 and bf16)
  }
  float* x0 = c->acts[0].x;
  RT_OTHER(1, rt::embed_gather(c->params, c->cur->tokens, x0, M, D, V, c->d_err, c->stream), "embed gather");
  float* x = x0;
  for (int l = 0; l < cfg.nlayers; ++l) {
    if (pend) cudaStreamWaitEvent(c->stream, c->ev_gather_seg[1 + l], 0);
    const rt::LayerActs& A = forward_only(c) ? c->acts[0] : c->acts[l];
    float* x_next;
    if (forward_only(c))
      x_next = (l + 1 == cfg.nlayers) ? c->x_out : (x == c->acts[0].x ? c->dy_a : c->acts[0].x);
    else
      x_next = (l + 1 == cfg.nlayers) ? c->x_out : c->acts[l + 1].x;
    if ((rc = layer_forward(c, l, A, x, x_next, batch))) return rc;
    x = x_next;
  }
  const float* gf = gamma_base(c);  // gamma_final sits first among the gammas
  RT_OTHER(1, rt::rmsnorm_fwd(c->x_out, gf, c->xf, c->rms_f, M, D, c->stream), "final rmsnorm");
  {  // tied-embedding logits (full_model.rs:228-230)
    rt::GemmArgs g;
    g.a = c->xf; g.lda = D;
    g.b = c->params_bf16; g.ldb = D; g.b_mn = false;
    g.M = M; g.N = V; g.K = D;
    g.epi = rt::kEpiF32; g.out = c->logits; g.ldo = V;
    if ((rc = gemm(c, g, "logits"))) return rc;
  }
  c->dl_ready = c->fuse_ce && !forward_only(c);
  c->fuse_ce = false;
  if (c->dl_ready)  // train step: loss and dlogits (full_model.rs:265-276) in one read of the logits
    RT_OTHER(1, rt::ce_fused(c->logits, c->cur->targets, c->row_loss, c->row_lse, c->dl, M, V, softcap,
                             c->fuse_ce_scale, c->stream),
             "ce fwd+bwd");
  else
    RT_OTHER(1, rt::ce_forward(c->logits, c->cur->targets, c->row_loss, c->row_lse, M, V, softcap, c->stream),
             "ce fwd");
  RT_OTHER(1, rt::mean_reduce(c->row_loss, M, c->d_loss, c->stream), "loss mean");
  if (pend) c->gather_pending = false;  // every segment has been waited for
  cudaEventRecord(c->ev[1], c->stream);
  c->ev_recorded |= 1u;
  c->cur_batch = batch;
  c->fwd_done = true;
  c->last_softcap = softcap;
  return RT_OK;
}

// --------------------------------------------------------------- backward
// Data-parallel all-reduce of one contiguous gradient range on the comm stream.
int allreduce_range(rt_ctx* c, int64_t begin, int64_t end, cudaStream_t st) {
  rt::NcclApi* api = rt::nccl_api();
  if (!api || !c->nccl || !c->nccl->comm) return set_err(c, RT_ERR_NCCL, "no communicator (aborted or not initialised)");
  ncclResult_t r = api->allReduce(c->grads + begin, c->grads + begin, static_cast<size_t>(end - begin), ncclFloat32,
                                  ncclSum, c->nccl->comm, st);
  if (r != ncclSuccess) return set_err(c, RT_ERR_NCCL, std::string("ncclAllReduce: ") + api->errorString(r));
  return RT_OK;
}

// ---- data-parallel sharding (see rt_ctx::zero)
int64_t seg_chunk(const rt_ctx* c, int i) { return (c->segs[i].second - c->segs[i].first) / c->world; }
int64_t seg_own(const rt_ctx* c, int i) { return c->segs[i].first + c->rank * seg_chunk(c, i); }

int nccl_ok(rt_ctx* c, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return RT_OK;
  return set_err(c, RT_ERR_NCCL, std::string(what) + ": " + rt::nccl_api()->errorString(r));
}

// Gradient segment i summed over the ranks into this rank's chunk (in place).
int reduce_scatter_seg(rt_ctx* c, int i, cudaStream_t st) {
  rt::NcclApi* api = rt::nccl_api();
  if (!api || !c->nccl || !c->nccl->comm) return set_err(c, RT_ERR_NCCL, "no communicator (aborted or not initialised)");
  float* base = c->grads + c->segs[i].first;
  return nccl_ok(c, api->reduceScatter(base, c->grads + seg_own(c, i), static_cast<size_t>(seg_chunk(c, i)),
                                       ncclFloat32, ncclSum, c->nccl->comm, st),
                 "ncclReduceScatter");
}

// Every rank's chunk of segment i of `arena` (fp32, or the bf16 copy) to all ranks (in place).
int gather_seg(rt_ctx* c, void* arena, bool bf16, int i, cudaStream_t st) {
  rt::NcclApi* api = rt::nccl_api();
  if (!api || !c->nccl || !c->nccl->comm) return set_err(c, RT_ERR_NCCL, "no communicator (aborted or not initialised)");
  const size_t es = bf16 ? 2 : 4;
  char* base = static_cast<char*>(arena) + c->segs[i].first * es;
  char* own = static_cast<char*>(arena) + seg_own(c, i) * es;
  return nccl_ok(c, api->allGather(own, base, static_cast<size_t>(seg_chunk(c, i)), bf16 ? ncclBfloat16 : ncclFloat32,
                                   c->nccl->comm, st),
                 "ncclAllGather");
}

// Gathers of several segments as one NCCL group.
template <class F>
int nccl_group(rt_ctx* c, F&& body) {
  rt::NcclApi* api = rt::nccl_api();
  if (api && api->groupStart) api->groupStart();
  const int rc = body();
  if (api && api->groupEnd) {
    const ncclResult_t r = api->groupEnd();
    if (rc == RT_OK && r != ncclSuccess) return nccl_ok(c, r, "ncclGroupEnd");
  }
  return rc;
}

// Collective: make the sharded arrays whole again on every rank (fp32 matrices
// and embedding / gammas, moments, gradients) before a call that reads them.
int zero_gather(rt_ctx* c, bool params, bool moments, bool grads) {
  join_gathers(c);
  const int nseg = static_cast<int>(c->segs.size());
  const bool gp = params && c->sharded_p, gm = moments && c->sharded_mv, gg = grads && c->sharded_g;
  if (!gp && !gm && !gg) return RT_OK;
  int rc = nccl_group(c, [&] {
    int r = RT_OK;
    for (int i = 0; i < nseg && r == RT_OK; ++i) {
      if (gp && i > 0 && i + 1 < nseg) r = gather_seg(c, c->params, false, i, c->stream);  // matrices
      if (r == RT_OK && gm) r = gather_seg(c, c->mom1, false, i, c->stream);
      if (r == RT_OK && gm) r = gather_seg(c, c->mom2, false, i, c->stream);
      if (r == RT_OK && gg) r = gather_seg(c, c->grads, false, i, c->stream);
    }
    return r;
  });
  if (rc) return rc;
  if (gp) c->sharded_p = false;
  if (gm) c->sharded_mv = false;
  if (gg) c->sharded_g = false;
  return RT_OK;
}

// Backward of the last forward.  The data-gradient chain (dlogits -> dx of each
// layer) runs on the main stream; each layer's four weight-gradient GEMMs run on
// s_dw as soon as their inputs exist, reading parity-double-buffered
// temporaries; with overlap_allreduce each layer's gradients are all-reduced on
// s_comm right after its weight-gradient GEMMs.  On return the main stream has
// waited for all of it.
// Backward of layer l (layer.rs:1606-1858): dy = gradient at the layer output
// (fp32), dffn[l & 1] = bf16(alpha * dy); writes dy_next = gradient at the layer
// input and, for l > 0, dffn[(l - 1) & 1] = bf16(alpha * dy_next).  Weight
// gradients go to the arena (beta = 0 overwrites) on the weight-gradient stream,
// whose last GEMM records ev_dw_done[l].
// Train step on one GPU: the weight-gradient GEMM k of layer l also writes its
// per-warp sums of squares of the final gradient, which the grad norm folds in
// instead of re-reading the layer's gradients.  (Data-parallel steps reduce the
// gradients across ranks first, so their norm reads the reduced values.)
void fold_sumsq(rt_ctx* c, rt::GemmArgs& g, int l, int k) {
  if (!c->layer_sumsq || c->overlap_allreduce) return;
  g.sumsq = c->gemm_sumsq + (int64_t(l) * 4 + k) * c->gemm_sumsq_slots;
  g.sumsq_slots = c->gemm_sumsq_slots;
}

int layer_backward(rt_ctx* c, int l, const float* dy, float* dy_next, int beta) {
  const auto& cfg = c->cfg;
  const int D = cfg.dim, H = cfg.hidden, S = cfg.seq, L = cfg.nlayers;
  const int batch = c->cur_batch, M = batch * S;
  const float alpha = alpha_of(cfg);
  const bf16* W = c->params_bf16;
  const float* P = c->params;
  float* Gr = c->grads;
  cudaStream_t ms = c->stream, ds = c->s_dw;
  int rc;
  const rt::LayerActs& A = c->acts[l];
  const auto& o = c->layer_off[l];
  const int p = l & 1;
  // the parity-p temporaries were last read by the weight GEMMs of layer l + 2
  if (l + 2 < L) cudaStreamWaitEvent(ms, c->ev_dw_done[l + 2], 0);
  {  // ffnBwdW2t + SiLU backward (layer.rs:1627-1667)
    rt::GemmArgs g;
    g.a = c->dffn[p]; g.lda = D;
    g.b = W + o.w2; g.ldb = H; g.b_mn = true;
    g.M = M; g.N = H; g.K = D;
    g.epi = rt::kEpiSwigluBwd; g.aux = A.h13; g.ld_aux = 2 * H; g.out = c->dh13[p]; g.ldo = 2 * H; g.n_half = H;
    if ((rc = gemm(c, g, "dgate"))) return rc;
  }
  cudaEventRecord(c->ev_dgate[l], ms);
  cudaStreamWaitEvent(ds, c->ev_dgate[l], 0);
  {  // dW2 += dffn^T gate (layer.rs:1754)
    rt::GemmArgs g;
    g.a = c->dffn[p]; g.lda = D; g.a_mn = true;
    g.b = A.gate; g.ldb = H; g.b_mn = true;
    g.M = D; g.N = H; g.K = M;
    g.epi = rt::kEpiF32Acc; g.out = Gr + o.w2; g.ldo = H; g.beta = beta;
    fold_sumsq(c, g, l, 0);
    if ((rc = gemm(c, g, "dW2", ds))) return rc;
  }
  {  // dW1 | dW3 += x2norm^T (dh1 | dh3) (layer.rs:1692, 1787)
    rt::GemmArgs g;
    g.a = A.x2n; g.lda = D; g.a_mn = true;
    g.b = c->dh13[p]; g.ldb = 2 * H; g.b_mn = true;
    g.M = D; g.N = 2 * H; g.K = M;
    g.epi = rt::kEpiF32Acc; g.out = Gr + o.w13; g.ldo = 2 * H; g.beta = beta;
    fold_sumsq(c, g, l, 1);
    if ((rc = gemm(c, g, "dW13", ds))) return rc;
  }
  {  // ffnBwdW13t: dx_ffn = dh1 W1^T + dh3 W3^T (layer.rs:1671-1699)
    rt::GemmArgs g;
    g.a = c->dh13[p]; g.lda = 2 * H;
    g.b = W + o.w13; g.ldb = 2 * H; g.b_mn = false;
    g.M = M; g.N = D; g.K = 2 * H;
    g.epi = rt::kEpiF32; g.out = c->dx_tmp; g.ldo = D;
    if ((rc = gemm(c, g, "dx_ffn"))) return rc;
  }
  // RMSNorm2 backward + dy (layer.rs:1702-1706); dx2s = alpha * dx2
  RT_OTHER(2, rt::rmsnorm_bwd(c->dx_tmp, A.x2, P + o.gamma2, A.rms2, dy, c->dx2, c->dx2s[p], alpha,
                              c->dgamma_part + (2 + 2 * l) * c->dgamma_stride, M, D, ms),
           "rmsnorm2 bwd");
  cudaEventRecord(c->ev_rms2[l], ms);
  cudaStreamWaitEvent(ds, c->ev_rms2[l], 0);
  {  // dWo += attn^T dx2s (layer.rs:1753)
    rt::GemmArgs g;
    g.a = A.attn; g.lda = cfg.q_dim; g.a_mn = true;
    g.b = c->dx2s[p]; g.ldb = D; g.b_mn = true;
    g.M = cfg.q_dim; g.N = D; g.K = M;
    g.epi = rt::kEpiF32Acc; g.out = Gr + o.wo; g.ldo = D; g.beta = beta;
    fold_sumsq(c, g, l, 2);
    if ((rc = gemm(c, g, "dWo", ds))) return rc;
  }
  {  // wotBwd: da = dx2s Wo^T (layer.rs:1709-1733)
    rt::GemmArgs g;
    g.a = c->dx2s[p]; g.lda = D;
    g.b = W + o.wo; g.ldb = D; g.b_mn = false;
    g.M = M; g.N = cfg.q_dim; g.K = D;
    g.out = c->da; g.ldo = cfg.q_dim;
    // the epilogue also writes the attention backward's rowsum(dO * O) per head
    g.epi = rt::kEpiBf16RowDot; g.aux = A.attn; g.ld_aux = cfg.q_dim; g.out2 = c->dvec; g.seq = S;
    if ((rc = gemm(c, g, "da"))) return rc;
  }
  {  // sdpaBwd1 + sdpaBwd2 + RoPE backward (layer.rs:1736-1798)
    rt::AttnArgs a;
    a.batch = batch; a.S = S; a.heads = cfg.heads; a.hd = cfg.hd; a.D = D;
    a.qkv = A.qkv; a.ldq = 3 * D; a.out = A.attn; a.ldo = D; a.lse2 = A.lse2;
    a.dout = c->da; a.lddo = D; a.dvec = c->dvec; a.dqkv = c->dqkv[p]; a.lddq = 3 * D;
    a.rope_cos_b = c->rope_cos_b; a.rope_sin_b = c->rope_sin_b; a.err = c->d_err; a.ds_scratch = c->attn_ds;
    a.dvec_ready = true;
    const double fl = 2.5 * 4.0 * batch * cfg.heads * double(S) * S / 2.0 * cfg.hd;
    RT_LAUNCH(launch(c, 1, fl, 3, [&] { return rt::attn_backward_tc(a, ms); }), "attention bwd");
  }
  cudaEventRecord(c->ev_attn[l], ms);
  cudaStreamWaitEvent(ds, c->ev_attn[l], 0);
  {  // dWq | dWk | dWv += xnorm^T (dq | dk | dv) (layer.rs:1838-1840)
    rt::GemmArgs g;
    g.a = A.xn; g.lda = D; g.a_mn = true;
    g.b = c->dqkv[p]; g.ldb = 3 * D; g.b_mn = true;
    g.M = D; g.N = 3 * D; g.K = M;
    g.epi = rt::kEpiF32Acc; g.out = Gr + o.wqkv; g.ldo = 3 * D; g.beta = beta;
    fold_sumsq(c, g, l, 3);
    if ((rc = gemm(c, g, "dWqkv", ds))) return rc;
  }
  cudaEventRecord(c->ev_dw_done[l], ds);
  {  // qBwd + kvBwd: dx_attn = dq Wq^T + dk Wk^T + dv Wv^T (layer.rs:1800-1850)
    rt::GemmArgs g;
    g.a = c->dqkv[p]; g.lda = 3 * D;
    g.b = W + o.wqkv; g.ldb = 3 * D; g.b_mn = false;
    g.M = M; g.N = D; g.K = 3 * D;
    g.epi = rt::kEpiF32; g.out = c->dx_tmp; g.ldo = D;
    if ((rc = gemm(c, g, "dx_attn"))) return rc;
  }
  // RMSNorm1 backward + dx2 (layer.rs:1853-1857); alpha * dx for the layer below, into the
  // other parity's dffn, last read by the weight GEMMs of layer l + 1
  if (l > 0 && l + 1 < L) cudaStreamWaitEvent(ms, c->ev_dw_done[l + 1], 0);
  RT_OTHER(2, rt::rmsnorm_bwd(c->dx_tmp, A.x, P + o.gamma1, A.rms1, c->dx2, dy_next,
                              l > 0 ? c->dffn[(l - 1) & 1] : nullptr, alpha,
                              c->dgamma_part + (1 + 2 * l) * c->dgamma_stride, M, D, ms),
           "rmsnorm1 bwd");
  return RT_OK;
}

// dgamma of `ngamma` adjacent gammas from their partial slots, one launch
// (slot 0 is the final norm's, at the arena's first gamma).
int reduce_dgammas(rt_ctx* c, int slot0, int ngamma, int beta) {
  const int M = c->cur_batch * c->cfg.seq, D = c->cfg.dim;
  RT_OTHER(1, rt::dgamma_reduce_many(c->dgamma_part + slot0 * c->dgamma_stride, c->dgamma_stride,
                                     rt::rmsnorm_bwd_blocks(M), c->grads + c->off_gamma_final + int64_t(slot0) * D, D,
                                     ngamma, beta, c->stream),
           "dgamma");
  return RT_OK;
}

int backward_impl(rt_ctx* c, float softcap, float loss_scale) {
  const auto& cfg = c->cfg;
  const int D = cfg.dim, H = cfg.hidden, V = cfg.vocab, S = cfg.seq, L = cfg.nlayers;
  const int batch = c->cur_batch, M = batch * S;
  const float alpha = alpha_of(cfg);
  const int beta = c->grads_zero_pending ? 0 : 1;
  const bf16* W = c->params_bf16;
  const float* P = c->params;
  float* Gr = c->grads;
  cudaStream_t ms = c->stream, ds = c->s_dw;
  int rc;
  cudaEventRecord(c->ev[2], ms);
  // dlogits * loss_scale (full_model.rs:265-276); CE mean over seq per sequence (cross_entropy.rs:92-95)
  if (!c->dl_ready)
    RT_OTHER(1, rt::ce_backward(c->logits, c->row_lse, c->cur->targets, c->dl, M, V, softcap, loss_scale / S, ms),
             "ce bwd");
  c->dl_ready = false;
  cudaEventRecord(c->ev_ce, ms);
  {  // dE += dl^T x_final   (full_model.rs:299-312) -- weight-gradient stream
    cudaStreamWaitEvent(ds, c->ev_ce, 0);
    rt::GemmArgs g;
    g.a = c->dl; g.lda = V; g.a_mn = true;
    g.b = c->xf; g.ldb = D; g.b_mn = true;
    g.M = V; g.N = D; g.K = M;
    g.epi = rt::kEpiF32Acc; g.out = Gr; g.ldo = D; g.beta = beta;
    if ((rc = gemm(c, g, "dE", ds))) return rc;
    cudaEventRecord(c->ev_de, ds);
  }
  {  // dx_final = dl * E   (full_model.rs:279-289)
    rt::GemmArgs g;
    g.a = c->dl; g.lda = V;
    g.b = W; g.ldb = D; g.b_mn = true;
    g.M = M; g.N = D; g.K = V;
    g.epi = rt::kEpiF32; g.out = c->dx_tmp; g.ldo = D;
    if ((rc = gemm(c, g, "dx_final"))) return rc;
  }
  // final RMSNorm backward (full_model.rs:315-318); also alpha*dy for the last layer
  RT_OTHER(2, rt::rmsnorm_bwd(c->dx_tmp, c->x_out, P + c->off_gamma_final, c->rms_f, nullptr, c->dy_a,
                              c->dffn[(L - 1) & 1], alpha, c->dgamma_part, M, D, ms),
           "final rmsnorm bwd");
  float* dy = c->dy_a;
  float* dy_next = c->dy_b;
  // Gradient segments that are final go to the comm stream: all-reduced (data
  // parallel) and / or reduced to grad-norm partials (train step), while the
  // backward continues.  Partials: [embed | layer 0 .. L-1 | gammas], SB each.
  const bool seg_norm = c->layer_sumsq;
  const int SB = rt::sumsq_seg_blocks();
  for (int l = L - 1; l >= 0; --l) {
    if ((rc = layer_backward(c, l, dy, dy_next, beta))) return rc;
    const auto& o = c->layer_off[l];
    if (c->overlap_allreduce || seg_norm) cudaStreamWaitEvent(c->s_comm, c->ev_dw_done[l], 0);
    const bool shard = c->overlap_allreduce && c->zero;
    if (c->overlap_allreduce) {  // this layer's matrices are final: reduce them while backward continues
      if (l == L - 1) cudaEventRecord(c->ev[4], c->s_comm);
      rc = shard ? reduce_scatter_seg(c, 1 + l, c->s_comm) : allreduce_range(c, o.wqkv, o.w2 + int64_t(D) * H, c->s_comm);
      if (rc) return rc;
    }
    if (seg_norm && !c->overlap_allreduce) {  // the layer's dW GEMMs wrote their sums of squares
      const int ns = 4 * c->gemm_sumsq_slots;
      RT_OTHER_ON(c->s_comm, 1,
                  rt::sumsq_fold(c->gemm_sumsq + int64_t(l) * ns, ns, c->norm_partials + (1 + l) * SB, SB, c->s_comm),
                  "grad norm");
    } else if (seg_norm) {  // sharded: this rank's chunk only (the ranks' sums are added after the backward)
      const int64_t b0 = shard ? seg_own(c, 1 + l) : o.wqkv;
      const int64_t n = shard ? seg_chunk(c, 1 + l) : o.w2 + int64_t(D) * H - o.wqkv;
      RT_OTHER_ON(c->s_comm, 1, rt::sumsq_partials(Gr + b0, n, c->norm_partials + (1 + l) * SB, c->s_comm),
                  "grad norm");
    }
    std::swap(dy, dy_next);
  }
  // dgamma of every RMSNorm from its partials in one launch (the gammas are the last
  // gradient segment; nothing reads them during the backward)
  if ((rc = reduce_dgammas(c, 0, 2 * L + 1, beta))) return rc;
  // embedding scatter-add (full_model.rs:330), after the dE GEMM
  cudaStreamWaitEvent(ms, c->ev_de, 0);
  RT_OTHER(1, rt::embed_scatter(dy, c->cur->perm, c->cur->seg_start, c->cur->seg_tok, c->cur->nseg, Gr, D, ms),
           "embed scatter");
  cudaStreamWaitEvent(ms, c->ev_dw_done[0], 0);  // every weight gradient is final
  if (c->overlap_allreduce || seg_norm) {  // last segments: embedding and the gammas
    cudaEventRecord(c->ev_main_done, ms);
    cudaStreamWaitEvent(c->s_comm, c->ev_main_done, 0);
    const bool shard = c->overlap_allreduce && c->zero;
    if (c->overlap_allreduce) {
      if (shard) {
        if ((rc = reduce_scatter_seg(c, 0, c->s_comm))) return rc;
        if ((rc = reduce_scatter_seg(c, L + 1, c->s_comm))) return rc;
      } else {
        if ((rc = allreduce_range(c, 0, c->n_embed, c->s_comm))) return rc;
        if ((rc = allreduce_range(c, c->n_matrix_end, c->n_params, c->s_comm))) return rc;
      }
      cudaEventRecord(c->ev[5], c->s_comm);
      c->ev_recorded |= 4u;
    }
    if (seg_norm) {
      const int64_t e0 = shard ? seg_own(c, 0) : 0, en = shard ? seg_chunk(c, 0) : c->n_embed;
      const int64_t g0 = shard ? seg_own(c, L + 1) : c->n_matrix_end;
      const int64_t gn = shard ? seg_chunk(c, L + 1) : c->n_params - c->n_matrix_end;
      RT_OTHER_ON(c->s_comm, 1, rt::sumsq_partials(Gr + e0, en, c->norm_partials, c->s_comm), "grad norm");
      RT_OTHER_ON(c->s_comm, 1, rt::sumsq_partials(Gr + g0, gn, c->norm_partials + int64_t(L + 1) * SB, c->s_comm),
                  "grad norm");
    }
    cudaEventRecord(c->ev_comm_all, c->s_comm);
    cudaStreamWaitEvent(ms, c->ev_comm_all, 0);
  }
  cudaEventRecord(c->ev[3], ms);
  c->ev_recorded |= 2u;
  c->grads_zero_pending = false;
  return RT_OK;
}

float powi_f32(float b, uint32_t t) {
  float r = 1.f;
  for (uint32_t i = 0; i < t; ++i) r *= b;
  return r;
}

int adam_impl(rt_ctx* c, uint32_t t, float lr, const rt_train_config* tc, float grad_scale, const float* d_norm,
              float gsc, float clip, bool shard = false, int only_seg = -1) {
  rt::AdamArgs a;
  a.param = c->params;
  a.grad = c->grads;
  a.m = c->mom1;
  a.v = c->mom2;
  a.param_bf16 = c->params_bf16;
  if (shard) {  // chunk `rank` of every gradient segment: embedding, layers, gammas
    const int nseg = static_cast<int>(c->segs.size());
    if (nseg > rt::kMaxAdamSegments) return set_err(c, RT_ERR_SHAPE, "too many segments for the sharded AdamW");
    a.nseg = 0;
    for (int i = 0; i < nseg; ++i) {
      if (only_seg >= 0 && i != only_seg) continue;
      const int64_t b = seg_own(c, i), e = b + seg_chunk(c, i);
      if (i == 0)
        a.seg[a.nseg++] = {b, e, lr * tc->embed_lr_scale, 0.f, 1};
      else if (i + 1 < nseg)
        a.seg[a.nseg++] = {b, e, lr * tc->matrix_lr_scale, tc->weight_decay, 1};
      else
        a.seg[a.nseg++] = {b, e, lr, 0.f, 0};
    }
  } else {
    a.nseg = 3;
    a.seg[0] = {0, c->n_embed, lr * tc->embed_lr_scale, 0.f, 1};
    a.seg[1] = {c->n_embed, c->n_matrix_end, lr * tc->matrix_lr_scale, tc->weight_decay, 1};
    a.seg[2] = {c->n_matrix_end, c->n_params, lr, 0.f, 0};
  }
  a.beta1 = tc->beta1;
  a.beta2 = tc->beta2;
  a.eps = tc->eps;
  a.bc1 = 1.0f / (1.0f - powi_f32(tc->beta1, t));
  a.bc2 = 1.0f / (1.0f - powi_f32(tc->beta2, t));
  a.grad_scale = grad_scale;
  a.norm = d_norm;
  a.gsc = gsc;
  a.clip = clip;
  RT_OTHER(1, rt::adam_step(a, c->stream), "adam");
  return RT_OK;
}

int check_train(rt_ctx* c) {
  if (!c) return RT_ERR_ARG;
  if (forward_only(c)) return set_err(c, RT_ERR_STATE, "context was created forward-only");
  return RT_OK;
}

}  // namespace

// ================================================================ C ABI
static thread_local std::string g_create_error;

extern "C" {

// rt_last_error(NULL) reports why the last rt_ctx_create on this thread failed.
RT_API const char* rt_last_error(const rt_ctx* c) { return c ? c->last_error.c_str() : g_create_error.c_str(); }

RT_API int rt_lcg_fill(float* out, int64_t n, float scale) {
  if (!out || n < 0) return RT_ERR_ARG;
  uint64_t seed = 42ull + static_cast<uint64_t>(n);  // crates/engine/src/layer.rs:404-413
  for (int64_t i = 0; i < n; ++i) {
    seed = seed * 6364136223846793005ull + 1442695040888963407ull;
    const float r =
        (static_cast<float>(static_cast<uint32_t>(seed >> 32)) / static_cast<float>(UINT32_MAX)) * 2.0f - 1.0f;
    out[i] = r * scale;
  }
  return RT_OK;
}

RT_API float rt_learning_rate(uint32_t step, const rt_train_config* tc) {
  if (!tc) return 0.f;
  if (step < tc->warmup_steps) return tc->max_lr * static_cast<float>(step + 1) / static_cast<float>(tc->warmup_steps);
  const float decay = static_cast<float>(step - tc->warmup_steps) / static_cast<float>(tc->total_steps - tc->warmup_steps);
  const float min_lr = tc->max_lr * tc->min_lr_frac;
  return min_lr + 0.5f * (1.0f + cosf(3.14159265358979323846f * decay)) * (tc->max_lr - min_lr);
}

RT_API int rt_ctx_create(const rt_model_config* cfgp, int device, int max_batch, int flags, rt_ctx** out) {
  if (!cfgp || !out || max_batch <= 0) return RT_ERR_ARG;
  *out = nullptr;
  const rt_model_config cfg = *cfgp;
  rt_ctx* c = new rt_ctx();
  c->cfg = cfg;
  c->device = device;
  c->max_batch = max_batch;
  c->flags = flags;
  auto bail = [&](int code, const std::string& msg) {
    g_create_error = msg;
    rt_ctx_destroy(c);
    return code;
  };
  if (cfg.hd != 128 || cfg.heads * cfg.hd != cfg.dim || cfg.q_dim != cfg.dim || cfg.kv_dim != cfg.dim ||
      cfg.kv_heads != cfg.heads || cfg.seq % 128 != 0 || cfg.dim % 128 != 0 || cfg.hidden % 64 != 0 ||
      cfg.vocab % 64 != 0 || cfg.nlayers <= 0 || cfg.dim > 8192 || cfg.vocab > 8192)
    return bail(RT_ERR_SHAPE, "unsupported model shape");
  if (cudaSetDevice(device) != cudaSuccess) return bail(RT_ERR_CUDA, "cudaSetDevice");
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) return bail(RT_ERR_CUDA, "stream");
  for (auto& e : c->ev) cudaEventCreate(&e);
  if (cudaStreamCreateWithFlags(&c->s_dw, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&c->s_comm, cudaStreamNonBlocking) != cudaSuccess)
    return bail(RT_ERR_CUDA, "streams");
  for (auto* v : {&c->ev_dgate, &c->ev_rms2, &c->ev_attn, &c->ev_dw_done, &c->ev_comm}) {
    v->resize(cfg.nlayers);
    for (auto& e : *v) cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
  }
  for (cudaEvent_t* e : {&c->ev_ce, &c->ev_de, &c->ev_main_done, &c->ev_comm_all})
    cudaEventCreateWithFlags(e, cudaEventDisableTiming);

  const int64_t D = cfg.dim, H = cfg.hidden, V = cfg.vocab, S = cfg.seq, L = cfg.nlayers, Q = cfg.q_dim;
  const int64_t M = int64_t(max_batch) * S;
  // parameter layout
  c->n_embed = V * D;
  int64_t off = c->n_embed;
  c->layer_off.resize(L);
  for (int64_t l = 0; l < L; ++l) {
    auto& o = c->layer_off[l];
    o.wqkv = off;
    off += D * 3 * D;
    o.wo = off;
    off += Q * D;
    o.w13 = off;
    off += D * 2 * H;
    o.w2 = off;
    off += D * H;
  }
  c->n_matrix_end = off;
  c->off_gamma_final = off;
  off += D;
  for (int64_t l = 0; l < L; ++l) {
    c->layer_off[l].gamma1 = off;
    off += D;
    c->layer_off[l].gamma2 = off;
    off += D;
  }
  c->n_params = off;

  const bool fo = (flags & RT_CTX_FORWARD_ONLY) != 0;
  bool ok = true;
  auto need = [&](void* p) {
    if (!p) ok = false;
  };
  c->d_err = dalloc<int>(c, 1);
  need(c->d_err);
  if (fo) {
    c->params = dalloc<float>(c, c->n_embed + (c->n_params - c->n_matrix_end));
    need(c->params);
  } else {
    c->params = dalloc<float>(c, c->n_params);
    c->grads = dalloc<float>(c, c->n_params);
    c->mom1 = dalloc<float>(c, c->n_params);
    c->mom2 = dalloc<float>(c, c->n_params);
    need(c->params);
    need(c->grads);
    need(c->mom1);
    need(c->mom2);
  }
  c->heads_loc = cfg.heads;
  c->head0 = 0;
  c->hid_loc = cfg.hidden;
  c->hid0 = 0;
  layout_bf16(c);
  const int nact = fo ? 1 : static_cast<int>(L);
  c->acts.resize(nact);
  for (auto& A : c->acts) {
    A.x = dalloc<float>(c, M * D);
    A.xn = dalloc<bf16>(c, M * D);
    A.rms1 = dalloc<float>(c, M);
    A.x2 = dalloc<float>(c, M * D);
    A.x2n = dalloc<bf16>(c, M * D);
    A.rms2 = dalloc<float>(c, M);
    for (void* p : {(void*)A.x, (void*)A.xn, (void*)A.rms1, (void*)A.x2, (void*)A.x2n, (void*)A.rms2}) need(p);
  }
  if (!alloc_shard_buffers(c)) ok = false;
  c->x_out = dalloc<float>(c, M * D);
  c->xf = dalloc<bf16>(c, M * D);
  c->rms_f = dalloc<float>(c, M);
  c->logits = dalloc<float>(c, M * V);
  c->row_loss = dalloc<float>(c, M);
  c->row_lse = dalloc<float>(c, M);
  c->d_loss = dalloc<float>(c, 4);
  c->d_norm = dalloc<float>(c, 4);
  c->norm_partials = dalloc<float>(
      c, std::max<int64_t>(rt::sumsq_partials_count(), int64_t(cfg.nlayers + 2) * rt::sumsq_seg_blocks()));
  c->dy_a = dalloc<float>(c, M * D);
  for (void* p : {(void*)c->x_out, (void*)c->xf, (void*)c->rms_f, (void*)c->logits, (void*)c->row_loss,
                  (void*)c->row_lse, (void*)c->d_loss, (void*)c->d_norm, (void*)c->norm_partials, (void*)c->dy_a})
    need(p);
  if (!fo) {
    c->gemm_sumsq_slots = rt::gemm_sumsq_slots();
    c->gemm_sumsq = dalloc<float>(c, int64_t(cfg.nlayers) * 4 * c->gemm_sumsq_slots);
    need(c->gemm_sumsq);
    c->dl = dalloc<bf16>(c, M * V);
    c->dy_b = dalloc<float>(c, M * D);
    c->dx_tmp = dalloc<float>(c, M * D);
    c->dx2 = dalloc<float>(c, M * D);
    for (int p = 0; p < 2; ++p) {
      c->dffn[p] = dalloc<bf16>(c, M * D);
      c->dx2s[p] = dalloc<bf16>(c, M * D);
      c->dh13[p] = dalloc<bf16>(c, M * 2 * H);
      c->dqkv[p] = dalloc<bf16>(c, M * 3 * D);
      need(c->dffn[p]);
      need(c->dx2s[p]);
      need(c->dh13[p]);
      need(c->dqkv[p]);
    }
    c->da = dalloc<bf16>(c, M * D);
    c->dvec = dalloc<float>(c, M * cfg.heads);
    c->attn_ds = dalloc<bf16>(c, static_cast<int64_t>(rt::attn_bwd_scratch_bytes(max_batch, S, cfg.heads) / 2));
    c->dgamma_stride = int64_t(rt::rmsnorm_bwd_blocks(static_cast<int>(M))) * D;
    c->dgamma_part = dalloc<float>(c, (2 * int64_t(cfg.nlayers) + 1) * c->dgamma_stride);
    for (void* p : {(void*)c->dl, (void*)c->dy_b, (void*)c->dx_tmp, (void*)c->dx2, (void*)c->da, (void*)c->dvec,
                    (void*)c->attn_ds, (void*)c->dgamma_part})
      need(p);
  }
  alloc_token_batch(c, c->io);
  c->rope_cos_f = dalloc<float>(c, S * 64);
  c->rope_sin_f = dalloc<float>(c, S * 64);
  c->rope_cos_b = dalloc<float>(c, S * 64);
  c->rope_sin_b = dalloc<float>(c, S * 64);
  for (void* p : {(void*)c->io.tokens, (void*)c->io.targets, (void*)c->io.perm, (void*)c->io.seg_start,
                  (void*)c->io.seg_tok, (void*)c->rope_cos_f, (void*)c->rope_sin_f, (void*)c->rope_cos_b,
                  (void*)c->rope_sin_b})
    need(p);
  if (!ok) return bail(RT_ERR_OOM, "device allocation failed");
  c->h_stage_bytes = sizeof(uint32_t) * (5 * M + 2);
  if (cudaMallocHost(&c->h_stage, c->h_stage_bytes) != cudaSuccess) return bail(RT_ERR_OOM, "pinned staging");
  if (cudaMallocHost(reinterpret_cast<void**>(&c->h_loss), 4 * sizeof(float)) != cudaSuccess)
    return bail(RT_ERR_OOM, "pinned loss");
  cudaMemset(c->d_err, 0, sizeof(int));
  std::vector<float> cf, sf, cb, sb;
  compute_rope_tables(cfg, cf, sf, cb, sb);
  cudaMemcpy(c->rope_cos_f, cf.data(), sizeof(float) * cf.size(), cudaMemcpyHostToDevice);
  cudaMemcpy(c->rope_sin_f, sf.data(), sizeof(float) * sf.size(), cudaMemcpyHostToDevice);
  cudaMemcpy(c->rope_cos_b, cb.data(), sizeof(float) * cb.size(), cudaMemcpyHostToDevice);
  cudaMemcpy(c->rope_sin_b, sb.data(), sizeof(float) * sb.size(), cudaMemcpyHostToDevice);
  if (cudaDeviceSynchronize() != cudaSuccess) return bail(RT_ERR_CUDA, "init");
  *out = c;
  return RT_OK;
}

RT_API int rt_ctx_destroy(rt_ctx* c) {
  if (!c) return RT_ERR_ARG;
  cudaSetDevice(c->device);
  if (c->nccl && c->nccl->comm) {
    // work still queued behind a collective whose peer has left would never finish:
    // give it the context's timeout, then abort the communicator so the streams drain
    rt::NcclApi* api = rt::nccl_api();
    const auto t0 = std::chrono::steady_clock::now();
    const int64_t limit_ms = std::max<int64_t>(c->timeout_ms, 1000);
    auto busy = [&] {
      for (cudaStream_t s : {c->stream, c->s_dw, c->s_comm})
        if (s && cudaStreamQuery(s) == cudaErrorNotReady) return true;
      return false;
    };
    while (busy()) {
      const auto ms =
          std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
      if (ms > limit_ms) {
        if (api) api->commAbort(c->nccl->comm);
        c->nccl->comm = nullptr;
        c->nccl->aborted = true;
        break;
      }
      std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
  }
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->s_dw) cudaStreamSynchronize(c->s_dw);
  if (c->s_comm) cudaStreamSynchronize(c->s_comm);
  if (c->nccl) {
    if (c->nccl->comm) {
      if (rt::NcclApi* api = rt::nccl_api()) api->commDestroy(c->nccl->comm);
    }
    delete c->nccl;
  }
  for (auto& a : c->allocations) cudaFree(a.first);
  if (c->h_stage) cudaFreeHost(c->h_stage);
  if (c->h_loss) cudaFreeHost(c->h_loss);
  for (auto& e : c->ev)
    if (e) cudaEventDestroy(e);
  for (auto e : c->event_pool) cudaEventDestroy(e);
  for (auto* v : {&c->ev_dgate, &c->ev_rms2, &c->ev_attn, &c->ev_dw_done, &c->ev_comm, &c->ev_adam_seg,
                  &c->ev_gather_seg})
    for (auto e : *v)
      if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : {c->ev_ce, c->ev_de, c->ev_main_done, c->ev_comm_all, c->ev_gather_all})
    if (e) cudaEventDestroy(e);
  if (c->s_dw) cudaStreamDestroy(c->s_dw);
  if (c->s_comm) cudaStreamDestroy(c->s_comm);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return RT_OK;
}

RT_API int rt_ctx_device_bytes(const rt_ctx* c, int64_t* out) {
  if (!c || !out) return RT_ERR_ARG;
  *out = c->device_bytes;
  return RT_OK;
}

RT_API int rt_weights_upload(rt_ctx* c, const rt_model_ptrs* w) {
  if (!c || !w) return RT_ERR_ARG;
  cudaSetDevice(c->device);
  join_gathers(c);
  const auto& cfg = c->cfg;
  const int64_t D = cfg.dim;
  int rc;
  if (!forward_only(c)) {
    if ((rc = arena_h2d(c, c->params, w))) return rc;
    RT_LAUNCH(rt::cast_bf16(c->params, c->params_bf16, c->n_matrix_end, c->stream), "cast bf16");
    c->weights_set = true;
    c->sharded_p = false;
  } else {
    // compact fp32 [embed | gammas]; this rank's matrix shard goes through a bounded fp32 staging buffer
    RT_CUDA(cudaMemcpyAsync(c->params, w->embed, sizeof(float) * c->n_embed, cudaMemcpyHostToDevice, c->stream), "upload embed");
    RT_LAUNCH(rt::cast_bf16(c->params, c->params_bf16, c->n_embed, c->stream), "cast bf16");
    float* gb = gamma_base(c);
    RT_CUDA(cudaMemcpyAsync(gb, w->gamma_final, sizeof(float) * D, cudaMemcpyHostToDevice, c->stream), "gamma_final");
    const int64_t H = cfg.hidden, Dl = int64_t(c->heads_loc) * cfg.hd, Hl = c->hid_loc;
    const int64_t q0 = int64_t(c->head0) * cfg.hd, h0 = c->hid0;
    const int64_t biggest = std::max<int64_t>(std::max<int64_t>(D * 3 * Dl, D * 2 * Hl), Dl * D);
    float* stage = nullptr;
    RT_CUDA(cudaMalloc(&stage, sizeof(float) * biggest), "staging");
    rc = 0;
    for (int l = 0; l < cfg.nlayers && rc == 0; ++l) {
      const auto& o = c->layer_off[l];
      const auto& ob = c->layer_off_b[l];
      const rt_layer_ptrs& L = w->layers[l];
      // Wq | Wk | Wv columns of this rank's heads
      if (!rc) rc = copy_block_h2d(c, stage, 3 * Dl, 0, L.wq + q0, D, Dl, D);
      if (!rc) rc = copy_block_h2d(c, stage, 3 * Dl, Dl, L.wk + q0, D, Dl, D);
      if (!rc) rc = copy_block_h2d(c, stage, 3 * Dl, 2 * Dl, L.wv + q0, D, Dl, D);
      if (!rc) rc = rt::cast_bf16(stage, c->params_bf16 + ob.wqkv, D * 3 * Dl, c->stream) ? RT_ERR_CUDA : 0;
      if (!rc) rc = cudaStreamSynchronize(c->stream) ? RT_ERR_CUDA : 0;
      // Wo rows of this rank's heads
      if (!rc) rc = cudaMemcpyAsync(stage, L.wo + q0 * D, sizeof(float) * Dl * D, cudaMemcpyHostToDevice, c->stream) ? RT_ERR_CUDA : 0;
      if (!rc) rc = rt::cast_bf16(stage, c->params_bf16 + ob.wo, Dl * D, c->stream) ? RT_ERR_CUDA : 0;
      if (!rc) rc = cudaStreamSynchronize(c->stream) ? RT_ERR_CUDA : 0;
      // W1 | W3 columns of this rank's hidden units
      if (!rc) rc = copy_block_h2d(c, stage, 2 * Hl, 0, L.w1 + h0, D, Hl, H);
      if (!rc) rc = copy_block_h2d(c, stage, 2 * Hl, Hl, L.w3 + h0, D, Hl, H);
      if (!rc) rc = rt::cast_bf16(stage, c->params_bf16 + ob.w13, D * 2 * Hl, c->stream) ? RT_ERR_CUDA : 0;
      if (!rc) rc = cudaStreamSynchronize(c->stream) ? RT_ERR_CUDA : 0;
      // W2 columns of this rank's hidden units
      if (!rc) rc = copy_block_h2d(c, stage, Hl, 0, L.w2 + h0, D, Hl, H);
      if (!rc) rc = rt::cast_bf16(stage, c->params_bf16 + ob.w2, D * Hl, c->stream) ? RT_ERR_CUDA : 0;
      if (!rc) rc = cudaStreamSynchronize(c->stream) ? RT_ERR_CUDA : 0;
      if (!rc) rc = cudaMemcpyAsync(gb + (o.gamma1 - c->n_matrix_end), L.gamma1, sizeof(float) * D, cudaMemcpyHostToDevice, c->stream)
                        ? RT_ERR_CUDA : 0;
      if (!rc) rc = cudaMemcpyAsync(gb + (o.gamma2 - c->n_matrix_end), L.gamma2, sizeof(float) * D, cudaMemcpyHostToDevice, c->stream)
                        ? RT_ERR_CUDA : 0;
    }
    cudaFree(stage);
    if (rc) return set_err(c, rc, "forward-only upload failed");
  }
  c->weights_set = true;
  RT_CUDA(cudaStreamSynchronize(c->stream), "upload sync");
  return RT_OK;
}

RT_API int rt_weights_download(rt_ctx* c, const rt_model_ptrs* w) {
  int rc;
  if ((rc = check_train(c))) return rc;
  cudaSetDevice(c->device);
  if ((rc = zero_gather(c, true, false, false))) return rc;
  RT_CUDA(cudaStreamSynchronize(c->stream), "sync");
  return arena_d2h(c, c->params, w);
}

RT_API int rt_grads_download(rt_ctx* c, const rt_model_ptrs* g) {
  int rc;
  if ((rc = check_train(c))) return rc;
  cudaSetDevice(c->device);
  if ((rc = materialize_zero_grads(c))) return rc;
  if ((rc = zero_gather(c, false, false, true))) return rc;
  RT_CUDA(cudaStreamSynchronize(c->stream), "sync");
  return arena_d2h(c, c->grads, g);
}

RT_API int rt_grads_upload(rt_ctx* c, const rt_model_ptrs* g) {
  int rc;
  if ((rc = check_train(c))) return rc;
  cudaSetDevice(c->device);
  join_gathers(c);
  RT_CUDA(cudaStreamSynchronize(c->stream), "sync");
  if ((rc = arena_h2d(c, c->grads, g))) return rc;
  c->grads_zero_pending = false;
  c->sharded_g = false;
  return RT_OK;
}

RT_API int rt_opt_download(rt_ctx* c, const rt_model_ptrs* m, const rt_model_ptrs* v) {
  int rc;
  if ((rc = check_train(c))) return rc;
  cudaSetDevice(c->device);
  if ((rc = zero_gather(c, false, true, false))) return rc;
  RT_CUDA(cudaStreamSynchronize(c->stream), "sync");
  if ((rc = arena_d2h(c, c->mom1, m))) return rc;
  return arena_d2h(c, c->mom2, v);
}

RT_API int rt_opt_upload(rt_ctx* c, const rt_model_ptrs* m, const rt_model_ptrs* v) {
  int rc;
  if ((rc = check_train(c))) return rc;
  cudaSetDevice(c->device);
  join_gathers(c);
  RT_CUDA(cudaStreamSynchronize(c->stream), "sync");
  if ((rc = arena_h2d(c, c->mom1, m))) return rc;
  c->sharded_mv = false;
  return arena_h2d(c, c->mom2, v);
}

RT_API int rt_weights_init_normal(rt_ctx* c, uint64_t seed, float std) {
  if (!c) return RT_ERR_ARG;
  cudaSetDevice(c->device);
  join_gathers(c);
  const int64_t D = c->cfg.dim;
  const int64_t n_gam = c->n_params - c->n_matrix_end;
  if (!forward_only(c)) {
    RT_LAUNCH(rt::init_normal(c->params, c->n_matrix_end, seed, std, c->stream), "init normal");
    RT_LAUNCH(rt::fill_f32(c->params + c->n_matrix_end, n_gam, 1.0f, c->stream), "init gammas");
    RT_LAUNCH(rt::cast_bf16(c->params, c->params_bf16, c->n_matrix_end, c->stream), "cast bf16");
    RT_CUDA(cudaMemsetAsync(c->mom1, 0, sizeof(float) * c->n_params, c->stream), "zero m");
    RT_CUDA(cudaMemsetAsync(c->mom2, 0, sizeof(float) * c->n_params, c->stream), "zero v");
    c->grads_zero_pending = true;
    c->sharded_p = c->sharded_mv = c->sharded_g = false;
  } else {
    // embed straight into the compact fp32 buffer; each matrix shard is generated at
    // the global indices of the full arena (same values as a training context / any TP degree)
    RT_LAUNCH(rt::init_normal(c->params, c->n_embed, seed, std, c->stream), "init embed");
    RT_LAUNCH(rt::fill_f32(gamma_base(c), n_gam, 1.0f, c->stream), "init gammas");
    RT_LAUNCH(rt::cast_bf16(c->params, c->params_bf16, c->n_embed, c->stream), "cast embed");
    const auto& cfg = c->cfg;
    const int64_t H = cfg.hidden, Dl = int64_t(c->heads_loc) * cfg.hd, Hl = c->hid_loc;
    const int64_t q0 = int64_t(c->head0) * cfg.hd, h0 = c->hid0;
    const int64_t biggest = std::max<int64_t>(std::max<int64_t>(D * 3 * Dl, D * 2 * Hl), Dl * D);
    float* stage = nullptr;
    RT_CUDA(cudaMalloc(&stage, sizeof(float) * biggest), "staging");
    int rc = 0;
    auto blk = [&](float* dst, int64_t rows, int64_t cols, int64_t dst_ld, int64_t gbase, int64_t gld, int64_t gcol0) {
      if (rc) return;
      rc = rt::init_normal_block(dst, rows, cols, dst_ld, gbase, gld, gcol0, seed, std, c->stream) ? RT_ERR_CUDA : 0;
    };
    for (int l = 0; l < cfg.nlayers && rc == 0; ++l) {
      const auto& o = c->layer_off[l];
      const auto& ob = c->layer_off_b[l];
      blk(stage, D, Dl, 3 * Dl, o.wqkv, 3 * D, q0);
      blk(stage + Dl, D, Dl, 3 * Dl, o.wqkv, 3 * D, D + q0);
      blk(stage + 2 * Dl, D, Dl, 3 * Dl, o.wqkv, 3 * D, 2 * D + q0);
      if (!rc) rc = rt::cast_bf16(stage, c->params_bf16 + ob.wqkv, D * 3 * Dl, c->stream) ? RT_ERR_CUDA : 0;
      blk(stage, Dl, D, D, o.wo + q0 * D, D, 0);
      if (!rc) rc = rt::cast_bf16(stage, c->params_bf16 + ob.wo, Dl * D, c->stream) ? RT_ERR_CUDA : 0;
      blk(stage, D, Hl, 2 * Hl, o.w13, 2 * H, h0);
      blk(stage + Hl, D, Hl, 2 * Hl, o.w13, 2 * H, H + h0);
      if (!rc) rc = rt::cast_bf16(stage, c->params_bf16 + ob.w13, D * 2 * Hl, c->stream) ? RT_ERR_CUDA : 0;
      blk(stage, D, Hl, Hl, o.w2, H, h0);
      if (!rc) rc = rt::cast_bf16(stage, c->params_bf16 + ob.w2, D * Hl, c->stream) ? RT_ERR_CUDA : 0;
      if (!rc) rc = cudaStreamSynchronize(c->stream) ? RT_ERR_CUDA : 0;
    }
    cudaFree(stage);
    if (rc) return set_err(c, RT_ERR_CUDA, "init normal (forward-only)");
  }
  c->weights_set = true;
  (void)D;
  RT_CUDA(cudaStreamSynchronize(c->stream), "init sync");
  return RT_OK;
}

RT_API int rt_forward(rt_ctx* c, const uint32_t* tokens, const uint32_t* targets, int batch, float softcap,
                      float* loss_out, float* per_token_loss) {
  if (!c || !tokens || !targets) return RT_ERR_ARG;
  if (batch <= 0 || batch > c->max_batch) return set_err(c, RT_ERR_SHAPE, "batch exceeds the context's max_batch");
  cudaSetDevice(c->device);
  int rc;
  if ((rc = upload_tokens(c, c->io, tokens, targets, batch))) return rc;
  c->cur = &c->io;
  if ((rc = forward_impl(c, batch, softcap))) return rc;
  RT_CUDA(cudaMemcpyAsync(c->h_loss, c->d_loss, sizeof(float), cudaMemcpyDeviceToHost, c->stream), "loss d2h");
  if ((rc = wait_stream(c))) return rc;
  if (loss_out) *loss_out = c->h_loss[0];
  if (per_token_loss)
    RT_CUDA(cudaMemcpyAsync(per_token_loss, c->row_loss, sizeof(float) * batch * c->cfg.seq, cudaMemcpyDeviceToHost, c->stream),
            "per-token loss");
  if (!std::isfinite(c->h_loss[0])) return set_err(c, RT_ERR_NONFINITE, "loss is not finite");
  return RT_OK;
}

RT_API int rt_logits_download(rt_ctx* c, float* logits) {
  if (!c || !logits) return RT_ERR_ARG;
  if (!c->fwd_done) return set_err(c, RT_ERR_STATE, "no forward pass yet");
  cudaSetDevice(c->device);
  const int64_t M = int64_t(c->cur_batch) * c->cfg.seq, V = c->cfg.vocab;
  RT_CUDA(cudaStreamSynchronize(c->stream), "sync");
  if (c->last_softcap > 0.f) {  // report the capped logits, as the reference stores them
    std::vector<float> h(M * V);
    RT_CUDA(cudaMemcpyAsync(h.data(), c->logits, sizeof(float) * M * V, cudaMemcpyDeviceToHost, c->stream), "logits");
    const float sc = c->last_softcap;
    for (int64_t i = 0; i < M * V; ++i) logits[i] = sc * tanhf(h[i] * (1.0f / sc));
    return RT_OK;
  }
  RT_CUDA(cudaMemcpyAsync(logits, c->logits, sizeof(float) * M * V, cudaMemcpyDeviceToHost, c->stream), "logits");
  return RT_OK;
}

RT_API int rt_backward(rt_ctx* c, float softcap, float loss_scale) {
  int rc;
  if ((rc = check_train(c))) return rc;
  if (!c->fwd_done) return set_err(c, RT_ERR_STATE, "backward before forward");
  cudaSetDevice(c->device);
  // accumulating into gradients a sharded train step left: make them whole first
  if (!c->grads_zero_pending && (rc = zero_gather(c, false, false, true))) return rc;
  if ((rc = backward_impl(c, softcap, loss_scale))) return rc;
  if (c->grads_zero_pending) c->sharded_g = false;
  return wait_stream(c);
}

RT_API int rt_grads_zero(rt_ctx* c) {
  int rc;
  if ((rc = check_train(c))) return rc;
  c->grads_zero_pending = true;
  return RT_OK;
}

RT_API int rt_grad_norm(rt_ctx* c, float* norm_out) {
  int rc;
  if ((rc = check_train(c))) return rc;
  cudaSetDevice(c->device);
  if ((rc = materialize_zero_grads(c))) return rc;
  if ((rc = zero_gather(c, false, false, true))) return rc;
  RT_OTHER(2, rt::sumsq_norm(c->grads, c->n_params, c->norm_partials, c->d_norm, c->stream), "grad norm");
  RT_CUDA(cudaMemcpyAsync(c->h_loss + 1, c->d_norm, sizeof(float), cudaMemcpyDeviceToHost, c->stream), "norm d2h");
  if ((rc = wait_stream(c))) return rc;
  c->norm_valid = true;
  if (norm_out) *norm_out = c->h_loss[1];
  return RT_OK;
}

RT_API int rt_last_grad_norm(rt_ctx* c, float* norm_out) {
  int rc;
  if ((rc = check_train(c))) return rc;
  if (!norm_out) return set_err(c, RT_ERR_ARG, "null argument");
  if (!c->norm_valid) return set_err(c, RT_ERR_STATE, "no gradient norm computed yet");
  cudaSetDevice(c->device);
  RT_CUDA(cudaMemcpyAsync(c->h_loss + 1, c->d_norm, sizeof(float), cudaMemcpyDeviceToHost, c->stream), "norm d2h");
  if ((rc = wait_stream(c))) return rc;
  *norm_out = c->h_loss[1];
  return RT_OK;
}

RT_API int rt_clip_grads(rt_ctx* c, float max_norm) {
  float norm = 0.f;
  int rc;
  if ((rc = rt_grad_norm(c, &norm))) return rc;
  if (norm > max_norm) {
    RT_OTHER(1, rt::scale_f32(c->grads, c->grads, c->n_params, max_norm / norm, c->stream), "clip");
    return wait_stream(c);
  }
  return RT_OK;
}

RT_API int rt_update_weights(rt_ctx* c, uint32_t t, float lr, const rt_train_config* tc, float grad_scale) {
  int rc;
  if ((rc = check_train(c))) return rc;
  if (!tc || t == 0) return set_err(c, RT_ERR_ARG, "train config missing or t == 0");
  cudaSetDevice(c->device);
  if ((rc = materialize_zero_grads(c))) return rc;
  if ((rc = zero_gather(c, true, true, true))) return rc;
  cudaEventRecord(c->ev[6], c->stream);
  if ((rc = adam_impl(c, t, lr, tc, grad_scale, nullptr, 0.f, 0.f))) return rc;
  cudaEventRecord(c->ev[7], c->stream);
  c->ev_recorded |= 8u;
  return wait_stream(c);
}

// ================================================================= single layer
namespace {

// [batch][D][S] (reference, channel-first) <-> [batch * S][D] (token-major)
void cf_to_tm(const float* cf, float* tm, int batch, int D, int S) {
  for (int b = 0; b < batch; ++b)
    for (int d = 0; d < D; ++d)
      for (int s = 0; s < S; ++s) tm[(int64_t(b) * S + s) * D + d] = cf[(int64_t(b) * D + d) * S + s];
}
void tm_to_cf(const float* tm, float* cf, int batch, int D, int S) {
  for (int b = 0; b < batch; ++b)
    for (int d = 0; d < D; ++d)
      for (int s = 0; s < S; ++s) cf[(int64_t(b) * D + d) * S + s] = tm[(int64_t(b) * S + s) * D + d];
}

int check_layer(rt_ctx* c, int layer) {
  int rc;
  if ((rc = check_train(c))) return rc;
  if (layer < 0 || layer >= c->cfg.nlayers) return set_err(c, RT_ERR_ARG, "layer index out of range");
  if (!c->weights_set) return set_err(c, RT_ERR_STATE, "weights not uploaded");
  if (c->tp) return set_err(c, RT_ERR_STATE, "single-layer calls run on unsharded contexts");
  cudaSetDevice(c->device);
  return zero_gather(c, true, true, true);  // a sharded data-parallel step left them in chunks (collective)
}

// Forward of layer `l` on host input x (reference layout); output left in c->x_out.
int layer_forward_host(rt_ctx* c, int l, const float* x, int batch) {
  const int D = c->cfg.dim, S = c->cfg.seq;
  const int64_t n = int64_t(batch) * S * D;
  std::vector<float> h(n);
  cf_to_tm(x, h.data(), batch, D, S);
  const rt::LayerActs& A = c->acts[l];
  RT_CUDA(cudaMemcpyAsync(A.x, h.data(), sizeof(float) * n, cudaMemcpyHostToDevice, c->stream), "layer input");
  int rc;
  if ((rc = layer_forward(c, l, A, A.x, c->x_out, batch))) return rc;
  c->cur_batch = batch;
  c->fwd_done = false;  // the model-level activations of layer l were overwritten
  c->layer_fwd = l;
  RT_CUDA(cudaStreamSynchronize(c->stream), "layer forward");  // h is read by the async copy
  return RT_OK;
}

// Backward of layer `l` from the device gradient c->dy_a; dx into c->dy_b; both streams joined.
int layer_backward_dev(rt_ctx* c, int l, int beta) {
  const int64_t n = int64_t(c->cur_batch) * c->cfg.seq * c->cfg.dim;
  RT_OTHER(1, rt::cast_bf16_scaled(c->dy_a, c->dffn[l & 1], n, alpha_of(c->cfg), c->stream), "alpha * dy");
  int rc;
  if ((rc = layer_backward(c, l, c->dy_a, c->dy_b, beta))) return rc;
  if ((rc = reduce_dgammas(c, 1 + 2 * l, 2, beta))) return rc;
  cudaStreamWaitEvent(c->stream, c->ev_dw_done[l], 0);
  return RT_OK;
}

}  // namespace

RT_API int rt_layer_forward(rt_ctx* c, int layer, const float* x, int batch, float* y) {
  int rc;
  if ((rc = check_layer(c, layer))) return rc;
  if (!x || !y) return set_err(c, RT_ERR_ARG, "null buffer");
  if (batch <= 0 || batch > c->max_batch) return set_err(c, RT_ERR_SHAPE, "batch exceeds the context's max_batch");
  cudaSetDevice(c->device);
  if ((rc = layer_forward_host(c, layer, x, batch))) return rc;
  const int D = c->cfg.dim, S = c->cfg.seq;
  std::vector<float> h(int64_t(batch) * S * D);
  RT_CUDA(cudaMemcpyAsync(h.data(), c->x_out, sizeof(float) * h.size(), cudaMemcpyDeviceToHost, c->stream), "y");
  if ((rc = wait_stream(c))) return rc;
  tm_to_cf(h.data(), y, batch, D, S);
  return RT_OK;
}

RT_API int rt_layer_backward(rt_ctx* c, int layer, const float* dy, float* dx) {
  int rc;
  if ((rc = check_layer(c, layer))) return rc;
  if (!dy || !dx) return set_err(c, RT_ERR_ARG, "null buffer");
  if (c->layer_fwd != layer) return set_err(c, RT_ERR_STATE, "rt_layer_backward without rt_layer_forward of the layer");
  cudaSetDevice(c->device);
  if ((rc = materialize_zero_grads(c))) return rc;  // accumulate semantics from here on
  const int batch = c->cur_batch, D = c->cfg.dim, S = c->cfg.seq;
  const int64_t n = int64_t(batch) * S * D;
  std::vector<float> h(n);
  cf_to_tm(dy, h.data(), batch, D, S);
  RT_CUDA(cudaMemcpyAsync(c->dy_a, h.data(), sizeof(float) * n, cudaMemcpyHostToDevice, c->stream), "dy");
  if ((rc = layer_backward_dev(c, layer, 1))) return rc;
  RT_CUDA(cudaMemcpyAsync(h.data(), c->dy_b, sizeof(float) * n, cudaMemcpyDeviceToHost, c->stream), "dx");
  if ((rc = wait_stream(c))) return rc;
  tm_to_cf(h.data(), dx, batch, D, S);
  return RT_OK;
}

RT_API int rt_layer_train_step(rt_ctx* c, int layer, const float* x, int batch, uint32_t t,
                               const rt_adam_config* ac, float* loss_out) {
  int rc;
  if ((rc = check_layer(c, layer))) return rc;
  if (!x || !ac || t == 0) return set_err(c, RT_ERR_ARG, "null input / config or t == 0");
  if (batch <= 0 || batch > c->max_batch) return set_err(c, RT_ERR_SHAPE, "batch exceeds the context's max_batch");
  cudaSetDevice(c->device);
  if ((rc = materialize_zero_grads(c))) return rc;  // other layers keep their (zero) gradients
  if ((rc = layer_forward_host(c, layer, x, batch))) return rc;
  const int64_t n = int64_t(batch) * c->cfg.seq * c->cfg.dim;
  // loss = mean(y^2) through the fixed-order L2 norm; dy = 2 y / n
  c->norm_valid = false;  // d_norm now holds the layer loss
  RT_OTHER(2, rt::sumsq_norm(c->x_out, n, c->norm_partials, c->d_norm, c->stream), "layer loss");
  RT_OTHER(1, rt::scale_f32(c->x_out, c->dy_a, n, 2.0f / static_cast<float>(n), c->stream), "dy");
  // grads.zero_out() of this layer: its weight gradients are overwritten (beta = 0)
  if ((rc = layer_backward_dev(c, layer, 0))) return rc;
  const auto& o = c->layer_off[layer];
  const int64_t D = c->cfg.dim, H = c->cfg.hidden;
  rt::AdamArgs a;
  a.param = c->params;
  a.grad = c->grads;
  a.m = c->mom1;
  a.v = c->mom2;
  a.param_bf16 = c->params_bf16;
  a.nseg = 3;
  a.seg[0] = {o.wqkv, o.w2 + D * H, ac->lr, ac->weight_decay, 1};
  a.seg[1] = {o.gamma1, o.gamma1 + D, ac->lr, ac->weight_decay, 0};
  a.seg[2] = {o.gamma2, o.gamma2 + D, ac->lr, ac->weight_decay, 0};
  a.beta1 = ac->beta1;
  a.beta2 = ac->beta2;
  a.eps = ac->eps;
  a.bc1 = 1.0f / (1.0f - powi_f32(ac->beta1, t));
  a.bc2 = 1.0f / (1.0f - powi_f32(ac->beta2, t));
  a.grad_scale = 1.0f;
  RT_OTHER(1, rt::adam_step(a, c->stream), "layer adam");
  float norm = 0.f;
  RT_CUDA(cudaMemcpyAsync(&norm, c->d_norm, sizeof(float), cudaMemcpyDeviceToHost, c->stream), "loss");
  if ((rc = wait_stream(c))) return rc;
  const float loss = norm * norm / static_cast<float>(n);
  if (loss_out) *loss_out = loss;
  if (!std::isfinite(loss)) return set_err(c, RT_ERR_NONFINITE, "loss is not finite");
  return RT_OK;
}

// Everything of train_step after the batch is on the device; async unless
// loss_out is given (then the loss is copied back and the stream waited on).
static int train_step_device(rt_ctx* c, const rt::TokenBatch& tb, uint32_t step, const rt_train_config* tc,
                             float* loss_out) {
  int rc;
  const int batch = tb.batch;
  c->cur = &tb;
  c->grads_zero_pending = true;  // grads.zero_out() (full_model.rs:675)
  c->fuse_ce = true;  // the backward below always follows: dlogits come out of the forward's CE pass
  c->fuse_ce_scale = tc->loss_scale / static_cast<float>(c->cfg.seq);
  if ((rc = forward_impl(c, batch, tc->softcap))) return rc;
  // data parallel: gradients are all-reduced bucket by bucket inside the backward
  c->overlap_allreduce = c->world > 1 && c->dist_mode == RT_DIST_DATA_PARALLEL;
  const bool shard = c->overlap_allreduce && c->zero;
  c->layer_sumsq = true;  // grad-norm partials of each segment as soon as it is final
  rc = backward_impl(c, tc->softcap, tc->loss_scale);
  c->overlap_allreduce = false;
  c->layer_sumsq = false;
  if (rc) return rc;
  cudaEventRecord(c->ev[6], c->stream);
  const int nparts = (c->cfg.nlayers + 2) * rt::sumsq_seg_blocks();
  if (shard) {  // this rank's sum of squares, summed over the ranks, then the square root
    RT_OTHER(1, rt::sumsq_finish_sq(c->norm_partials, nparts, c->d_sumsq, c->stream), "grad norm");
    if ((rc = nccl_ok(c, rt::nccl_api()->allReduce(c->d_sumsq, c->d_sumsq, 1, ncclFloat64, ncclSum, c->nccl->comm,
                                                   c->stream),
                      "ncclAllReduce")))
      return rc;
    RT_OTHER(1, rt::sqrt_to_float(c->d_sumsq, c->d_norm, c->stream), "grad norm");
  } else {
    RT_OTHER(1, rt::sumsq_finish(c->norm_partials, nparts, c->d_norm, c->stream), "grad norm");
  }
  c->norm_valid = true;
  const float gsc = 1.0f / (static_cast<float>(batch) * static_cast<float>(c->world) * tc->loss_scale);
  const float lr = rt_learning_rate(step, tc);
  if (!shard) {
    if ((rc = adam_impl(c, step + 1, lr, tc, 1.0f, c->d_norm, gsc, tc->grad_clip))) return rc;
  } else {
    // AdamW segment by segment in the order the next forward needs the weights
    // (gammas, embedding, layers), each followed on the comm stream by the
    // all-gather of what the forward reads: fp32 gammas, fp32 + bf16 embedding,
    // bf16 layer matrices.  The next forward waits per segment.
    const int nseg = static_cast<int>(c->segs.size());
    for (int k = 0; k < nseg; ++k) {
      const int i = k == 0 ? nseg - 1 : k - 1;
      if ((rc = adam_impl(c, step + 1, lr, tc, 1.0f, c->d_norm, gsc, tc->grad_clip, true, i))) return rc;
      cudaEventRecord(c->ev_adam_seg[i], c->stream);
    }
    for (int k = 0; k < nseg; ++k) {
      const int i = k == 0 ? nseg - 1 : k - 1;
      cudaStreamWaitEvent(c->s_comm, c->ev_adam_seg[i], 0);
      rc = nccl_group(c, [&] {
        if (i == nseg - 1) return gather_seg(c, c->params, false, i, c->s_comm);
        int r = i == 0 ? gather_seg(c, c->params, false, 0, c->s_comm) : RT_OK;
        return r ? r : gather_seg(c, c->params_bf16, true, i, c->s_comm);
      });
      if (rc) return rc;
      cudaEventRecord(c->ev_gather_seg[i], c->s_comm);
    }
    cudaEventRecord(c->ev_gather_all, c->s_comm);
    c->gather_pending = true;
    c->sharded_p = c->sharded_mv = c->sharded_g = true;
  }
  cudaEventRecord(c->ev[7], c->stream);
  c->ev_recorded |= 8u;
  if (!loss_out) return RT_OK;
  RT_CUDA(cudaMemcpyAsync(c->h_loss, c->d_loss, sizeof(float), cudaMemcpyDeviceToHost, c->stream), "loss d2h");
  if ((rc = wait_stream(c))) return rc;
  *loss_out = c->h_loss[0];
  if (!std::isfinite(c->h_loss[0])) return set_err(c, RT_ERR_NONFINITE, "loss is not finite");
  return RT_OK;
}

RT_API int rt_train_step(rt_ctx* c, const uint32_t* tokens, const uint32_t* targets, int batch, uint32_t step,
                         const rt_train_config* tc, float* loss_out) {
  int rc;
  if ((rc = check_train(c))) return rc;
  if (!tokens || !targets || !tc) return set_err(c, RT_ERR_ARG, "null argument");
  if (batch <= 0 || batch > c->max_batch) return set_err(c, RT_ERR_SHAPE, "batch exceeds the context's max_batch");
  cudaSetDevice(c->device);
  if ((rc = upload_tokens(c, c->io, tokens, targets, batch))) return rc;
  float loss = 0.f;
  if ((rc = train_step_device(c, c->io, step, tc, &loss))) return rc;
  if (loss_out) *loss_out = loss;
  return RT_OK;
}

RT_API int rt_stage_batch(rt_ctx* c, int slot, const uint32_t* tokens, const uint32_t* targets, int batch) {
  if (!c || !tokens || !targets || slot < 0 || slot > 4095) return RT_ERR_ARG;
  if (batch <= 0 || batch > c->max_batch) return set_err(c, RT_ERR_SHAPE, "batch exceeds the context's max_batch");
  cudaSetDevice(c->device);
  if (static_cast<size_t>(slot) >= c->staged.size()) c->staged.resize(slot + 1);
  rt::TokenBatch& tb = c->staged[slot];
  if (!tb.tokens) {
    alloc_token_batch(c, tb);
    if (!tb.tokens || !tb.targets || !tb.perm || !tb.seg_start || !tb.seg_tok)
      return set_err(c, RT_ERR_OOM, "staged batch allocation");
  }
  int rc;
  if ((rc = upload_tokens(c, tb, tokens, targets, batch))) return rc;
  RT_CUDA(cudaStreamSynchronize(c->stream), "stage sync");
  return RT_OK;
}

RT_API int rt_train_step_staged(rt_ctx* c, int slot, uint32_t step, const rt_train_config* tc, float* loss_out) {
  int rc;
  if ((rc = check_train(c))) return rc;
  if (!tc || slot < 0 || static_cast<size_t>(slot) >= c->staged.size() || !c->staged[slot].tokens ||
      c->staged[slot].batch == 0)
    return set_err(c, RT_ERR_ARG, "no staged batch in that slot");
  cudaSetDevice(c->device);
  return train_step_device(c, c->staged[slot], step, tc, loss_out);
}

RT_API int rt_forward_staged(rt_ctx* c, int slot, float softcap) {
  if (!c || slot < 0 || static_cast<size_t>(slot) >= c->staged.size() || c->staged[slot].batch == 0)
    return RT_ERR_ARG;
  cudaSetDevice(c->device);
  c->cur = &c->staged[slot];
  return forward_impl(c, c->staged[slot].batch, softcap);
}

RT_API int rt_sync(rt_ctx* c, float* loss_out) {
  if (!c) return RT_ERR_ARG;
  cudaSetDevice(c->device);
  int rc;
  if (loss_out) RT_CUDA(cudaMemcpyAsync(c->h_loss, c->d_loss, sizeof(float), cudaMemcpyDeviceToHost, c->stream), "loss");
  if ((rc = wait_stream(c))) return rc;
  if (loss_out) *loss_out = c->h_loss[0];
  return RT_OK;
}

RT_API int rt_join(rt_ctx* c) {
  if (!c) return RT_ERR_ARG;
  cudaSetDevice(c->device);
  join_gathers(c);
  return RT_OK;
}

RT_API int rt_ctx_stream(const rt_ctx* c, void** stream_out) {
  if (!c || !stream_out) return RT_ERR_ARG;
  *stream_out = c->stream;
  return RT_OK;
}

RT_API int rt_last_h2d_bytes(const rt_ctx* c, int64_t* out) {
  if (!c || !out) return RT_ERR_ARG;
  *out = c->h2d_bytes_last;
  return RT_OK;
}

RT_API int rt_nccl_unique_id(uint8_t* out128) {
  if (!out128) return RT_ERR_ARG;
  rt::NcclApi* api = rt::nccl_api();
  if (!api) return RT_ERR_NCCL;
  ncclUniqueId id;
  if (api->getUniqueId(&id) != ncclSuccess) return RT_ERR_NCCL;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  memcpy(out128, &id, 128);
  return RT_OK;
}

RT_API int rt_tp_shard(int heads, int hidden, int world, int rank, int* head0, int* heads_loc, int* hid0,
                       int* hid_loc) {
  if (!head0 || !heads_loc || !hid0 || !hid_loc) return RT_ERR_ARG;
  if (world < 1 || rank < 0 || rank >= world || heads < world) return RT_ERR_SHAPE;
  if (world == 1) {
    *head0 = *hid0 = 0;
    *heads_loc = heads;
    *hid_loc = hidden;
    return RT_OK;
  }
  if (hidden % 64 != 0 || hidden / 64 < world) return RT_ERR_SHAPE;
  // heads: the first heads % world ranks take one extra; hidden columns likewise in 64-column units
  const int units = hidden / 64;
  const int hb = heads / world, hr = heads % world, ub = units / world, ur = units % world;
  *heads_loc = hb + (rank < hr ? 1 : 0);
  *head0 = rank * hb + std::min(rank, hr);
  *hid_loc = 64 * (ub + (rank < ur ? 1 : 0));
  *hid0 = 64 * (rank * ub + std::min(rank, ur));
  return RT_OK;
}

RT_API int rt_dist_init(rt_ctx* c, int world, int rank, const uint8_t* unique_id128, int mode, int timeout_ms) {
  if (!c || world <= 0 || rank < 0 || rank >= world) return RT_ERR_ARG;
  if (mode != RT_DIST_DATA_PARALLEL && mode != RT_DIST_TENSOR_PARALLEL) return RT_ERR_ARG;
  if (c->nccl) return set_err(c, RT_ERR_STATE, "rt_dist_init was already called on this context");
  const int nh = c->cfg.heads, units = c->cfg.hidden / 64;
  if (mode == RT_DIST_TENSOR_PARALLEL) {
    if (!forward_only(c)) return set_err(c, RT_ERR_STATE, "tensor parallelism needs a forward-only context");
    if (c->weights_set) return set_err(c, RT_ERR_STATE, "call rt_dist_init before uploading or initialising weights");
    if (world > nh || world > units || (world > 1 && c->cfg.hidden % 64 != 0))
      return set_err(c, RT_ERR_SHAPE, "more tensor-parallel ranks than heads or 64-column hidden units");
  }
  // join the communicator before changing the context, so that a failed join leaves it as it was
  rt::NcclApi* api = nullptr;
  if (world > 1) {
    if (!unique_id128) return RT_ERR_ARG;
    api = rt::nccl_api();
    if (!api) return set_err(c, RT_ERR_NCCL, "libnccl.so.2 could not be loaded");
    cudaSetDevice(c->device);
    ncclUniqueId id;
    memcpy(&id, unique_id128, 128);
    ncclComm_t comm = nullptr;
    ncclResult_t r = api->commInitRank(&comm, world, id, rank);
    if (r != ncclSuccess) return set_err(c, RT_ERR_NCCL, std::string("ncclCommInitRank: ") + api->errorString(r));
    c->nccl = new rt::NcclState();
    c->nccl->comm = comm;
  }
  if (mode == RT_DIST_TENSOR_PARALLEL) {
    free_shard_buffers(c);
    c->tp = world > 1;
    rt_tp_shard(nh, c->cfg.hidden, world, rank, &c->head0, &c->heads_loc, &c->hid0, &c->hid_loc);
    layout_bf16(c);
    if (!alloc_shard_buffers(c)) return set_err(c, RT_ERR_OOM, "tensor-parallel shard allocation");
  }
  c->world = world;
  c->rank = rank;
  c->dist_mode = mode;
  c->timeout_ms = timeout_ms;
  if (world == 1) return RT_OK;
  if (mode == RT_DIST_DATA_PARALLEL && !forward_only(c)) {
    // shard the optimizer when every gradient segment splits into 16-byte-aligned
    // chunks, one per rank (RUSTANE_DP_ALLREDUCE=1 keeps the all-reduce of every gradient)
    c->segs.clear();
    c->segs.push_back({0, c->n_embed});
    for (const auto& o : c->layer_off) c->segs.push_back({o.wqkv, o.w2 + int64_t(c->cfg.dim) * c->cfg.hidden});
    c->segs.push_back({c->n_matrix_end, c->n_params});
    bool ok = api->reduceScatter && api->allGather && !getenv("RUSTANE_DP_ALLREDUCE") &&
              static_cast<int>(c->segs.size()) <= rt::kMaxAdamSegments;
    for (const auto& sg : c->segs) ok = ok && (sg.second - sg.first) % (int64_t(4) * world) == 0;
    if (ok && !c->d_sumsq) c->d_sumsq = dalloc<double>(c, 1);
    if (ok && c->ev_adam_seg.empty()) {
      c->ev_adam_seg.resize(c->segs.size());
      c->ev_gather_seg.resize(c->segs.size());
      for (auto* v : {&c->ev_adam_seg, &c->ev_gather_seg})
        for (auto& e : *v) ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
      ok = ok && cudaEventCreateWithFlags(&c->ev_gather_all, cudaEventDisableTiming) == cudaSuccess;
    }
    c->zero = ok && c->d_sumsq;
    c->sharded_p = c->sharded_mv = c->sharded_g = false;
  }
  return RT_OK;
}

RT_API int rt_dist_ranks(const rt_ctx* c, int* nranks_out) {
  if (!c || !nranks_out) return RT_ERR_ARG;
  *nranks_out = 1;
  if (!c->nccl || !c->nccl->comm) return RT_OK;
  rt::NcclApi* api = rt::nccl_api();
  if (!api || !api->commCount) return RT_ERR_NCCL;
  int n = 0;
  if (api->commCount(c->nccl->comm, &n) != ncclSuccess) return RT_ERR_NCCL;
  *nranks_out = n;
  return RT_OK;
}

RT_API int rt_grad_allreduce(rt_ctx* c) {
  int rc;
  if ((rc = check_train(c))) return rc;
  if (c->world == 1) return RT_OK;
  if (!c->nccl || !c->nccl->comm) return set_err(c, RT_ERR_NCCL, "no communicator (aborted or not initialised)");
  if ((rc = materialize_zero_grads(c))) return rc;
  // after a sharded train step each rank holds the summed gradients of its chunks: gathering them is the sum
  if (c->sharded_g) return zero_gather(c, false, false, true);
  rt::NcclApi* api = rt::nccl_api();
  ncclResult_t r = api->allReduce(c->grads, c->grads, static_cast<size_t>(c->n_params), ncclFloat32, ncclSum,
                                  c->nccl->comm, c->stream);
  if (r != ncclSuccess) return set_err(c, RT_ERR_NCCL, std::string("ncclAllReduce: ") + api->errorString(r));
  return RT_OK;
}

RT_API int rt_profile(rt_ctx* c, int enable) {
  if (!c) return RT_ERR_ARG;
  cudaStreamSynchronize(c->stream);
  c->kevents.clear();
  c->event_pool_used = 0;
  const int64_t launches = c->acc.kernel_launches;
  c->acc = rt_timings{};
  c->acc.kernel_launches = launches;
  c->profiling = enable != 0;
  return RT_OK;
}

RT_API int rt_get_timings(rt_ctx* c, rt_timings* out) {
  if (!c || !out) return RT_ERR_ARG;
  cudaStreamSynchronize(c->stream);
  if (c->profiling) harvest_kernel_events(c);
  rt_timings t = c->acc;
  double* dst[4] = {&t.fwd_ms, &t.bwd_ms, &t.comm_ms, &t.opt_ms};
  for (int i = 0; i < 4; ++i) {
    float ms = 0.f;
    if ((c->ev_recorded >> i) & 1u) {
      if (cudaEventElapsedTime(&ms, c->ev[2 * i], c->ev[2 * i + 1]) == cudaSuccess) *dst[i] = ms;
      else cudaGetLastError();  // a pair still pending is not an error of the next launch
    }
  }
  *out = t;
  return RT_OK;
}

}  // extern "C"
