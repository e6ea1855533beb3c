// Internal runtime state of an rt_ctx (librustane_cuda).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <deque>
#include <string>
#include <vector>

#include "rustane_cuda.h"

namespace rt {

using bf16 = __nv_bfloat16;

// Offsets (elements) of one layer's tensors inside the parameter arena.
// Wqkv is [dim, 3*dim] with rows wq[i,:] | wk[i,:] | wv[i,:]; W13 is
// [dim, 2*hidden] with rows w1[i,:] | w3[i,:]; Wo [q_dim, dim]; W2 [dim, hidden].
struct LayerOffsets {
  int64_t wqkv, wo, w13, w2, gamma1, gamma2;
};

// Activations of one layer kept for the backward pass (token-major, M rows).
struct LayerActs {
  float* x = nullptr;      // [M, D] layer input (fp32 residual stream)
  bf16* xn = nullptr;      // [M, D] RMSNorm1 output
  float* rms1 = nullptr;   // [M]
  bf16* qkv = nullptr;     // [M, 3D] roped Q, K and V
  bf16* attn = nullptr;    // [M, D] attention output
  float* lse2 = nullptr;   // [B, heads, S]
  float* x2 = nullptr;     // [M, D] x + alpha * attn Wo
  bf16* x2n = nullptr;     // [M, D] RMSNorm2 output
  float* rms2 = nullptr;   // [M]
  bf16* h13 = nullptr;     // [M, 2H] h1 | h3
  bf16* gate = nullptr;    // [M, H] silu(h1) * h3
};

struct KernelEvent {
  int kind;  // 0 gemm, 1 attention, 2 other
  double flops;
  cudaEvent_t a, b;
};

struct NcclState;

// One batch of token ids on the device plus the embedding-scatter segments
// (positions grouped by token, ascending) built from it on the host.
struct TokenBatch {
  uint32_t* tokens = nullptr;
  uint32_t* targets = nullptr;
  int32_t* perm = nullptr;
  int32_t* seg_start = nullptr;
  uint32_t* seg_tok = nullptr;
  int nseg = 0;
  int batch = 0;
};

}  // namespace rt

struct rt_ctx {
  rt_model_config cfg{};
  int device = 0;
  int max_batch = 0;
  int flags = 0;
  cudaStream_t stream = nullptr;
  std::string last_error;
  int* d_err = nullptr;
  int layer_fwd = -1;  // layer of the last rt_layer_forward (its activations are cached)

  // parameter arenas (elements): [embed | matrices | gammas]
  int64_t n_params = 0, n_embed = 0, n_matrix_end = 0;
  int64_t off_gamma_final = 0;
  std::vector<rt::LayerOffsets> layer_off;
  float* params = nullptr;  // fp32 master (forward-only: gammas + embed only are meaningful)
  float* grads = nullptr;
  float* mom1 = nullptr;
  float* mom2 = nullptr;
  rt::bf16* params_bf16 = nullptr;  // [embed | matrices]

  // activations
  std::vector<rt::LayerActs> acts;
  float* x_out = nullptr;  // [M, D] final layer output (pre final norm)
  rt::bf16* xf = nullptr;  // [M, D] final-norm output
  float* rms_f = nullptr;  // [M]
  float* logits = nullptr;  // [M, V]
  float* row_loss = nullptr;
  float* row_lse = nullptr;
  float* d_loss = nullptr;  // [1]
  float* d_norm = nullptr;  // [1]
  // per layer and weight-gradient GEMM (dW2, dW13, dWo, dWqkv): the GEMM epilogue's
  // per-warp sums of squares of the final gradient (gemm_sumsq_slots floats each)
  float* gemm_sumsq = nullptr;
  int gemm_sumsq_slots = 0;
  bool norm_valid = false;  // d_norm holds the last computed gradient norm
  // train step: the forward's cross-entropy also writes dlogits (scale fuse_ce_scale),
  // so the backward that follows skips its own pass over the logits
  bool fuse_ce = false;
  float fuse_ce_scale = 0.f;
  bool dl_ready = false;
  float* norm_partials = nullptr;

  // backward scratch
  rt::bf16* dl = nullptr;    // [M, V]
  float* dy_a = nullptr;     // [M, D]
  float* dy_b = nullptr;     // [M, D]
  float* dx_tmp = nullptr;   // [M, D]
  float* dx2 = nullptr;      // [M, D]
  // Backward temporaries read by the weight-gradient GEMMs on the second
  // stream: two copies each, by layer parity, so the data-gradient chain of
  // layer l-1 can run while the weight gradients of layer l are computed.
  rt::bf16* dffn[2] = {};  // [M, D] alpha * dy
  rt::bf16* dx2s[2] = {};  // [M, D] alpha * dx2
  rt::bf16* dh13[2] = {};  // [M, 2H]
  rt::bf16* dqkv[2] = {};  // [M, 3D]
  rt::bf16* da = nullptr;  // [M, D]
  float* dvec = nullptr;     // [B, heads, S]
  rt::bf16* attn_ds = nullptr;  // dS^T tiles of the tcgen05 attention backward (B * heads * S * S)
  // RMSNorm dgamma partials, one slot of dgamma_stride floats per gamma in arena order
  // (slot 0 the final norm, 1 + 2l / 2 + 2l layer l's gamma1 / gamma2): the backward
  // reduces all of them in one launch after its last layer.
  float* dgamma_part = nullptr;
  int64_t dgamma_stride = 0;

  // tokens and the embedding-scatter segments: `io` is refilled by every call
  // that takes host tokens; `staged` slots hold batches uploaded ahead of time.
  rt::TokenBatch io;
  std::deque<rt::TokenBatch> staged;  // deque: growing keeps `cur` valid
  const rt::TokenBatch* cur = nullptr;  // batch used by the last / running forward
  void* h_stage = nullptr;  // pinned staging for token uploads
  size_t h_stage_bytes = 0;
  float* h_loss = nullptr;  // pinned

  // rope tables
  float* rope_cos_f = nullptr;  // [S][hd/2]
  float* rope_sin_f = nullptr;
  float* rope_cos_b = nullptr;  // [hd/2][S]
  float* rope_sin_b = nullptr;

  // state
  int cur_batch = 0;
  bool fwd_done = false;
  bool grads_zero_pending = true;
  float last_softcap = 0.f;
  int64_t device_bytes = 0;
  int64_t h2d_bytes_last = 0;
  std::vector<std::pair<void*, size_t>> allocations;

  // tensor parallelism (forward-only contexts): this rank's heads [head0, head0 + heads_loc)
  // and hidden columns [hid0, hid0 + hid_loc); without TP they are all heads / columns
  bool tp = false;
  int heads_loc = 0, head0 = 0, hid_loc = 0, hid0 = 0;
  std::vector<rt::LayerOffsets> layer_off_b;  // bf16 weight arena offsets (this rank's shard shapes)
  int64_t n_bf16 = 0;
  rt::bf16* tp_partial = nullptr;  // [M, D] bf16 partial sum of a row-parallel GEMM
  bool weights_set = false;

  // distributed
  int world = 1, rank = 0, dist_mode = -1, timeout_ms = 0;
  rt::NcclState* nccl = nullptr;
  // Data-parallel optimizer sharding: every gradient segment (embedding, each
  // layer's matrices, the gammas) is reduce-scattered, rank r runs AdamW on chunk r
  // of every segment, then the weights the forward reads (bf16 copy, fp32
  // embedding and gammas) are all-gathered.  The fp32 matrices, the moments and
  // the gradients stay sharded until a call that reads them whole gathers them.
  bool zero = false;
  bool sharded_p = false, sharded_mv = false, sharded_g = false;
  std::vector<std::pair<int64_t, int64_t>> segs;  // arena ranges [embed, layer 0 .. L-1, gammas]
  double* d_sumsq = nullptr;                      // [1] sum of squares of the gradients, all ranks
  // Sharded step tail: AdamW of segment i on the main stream records ev_adam_seg[i];
  // the comm stream gathers segment i after it and records ev_gather_seg[i]; the
  // next forward waits segment by segment (gather_pending), every other reader
  // waits for ev_gather_all.
  std::vector<cudaEvent_t> ev_adam_seg, ev_gather_seg;
  cudaEvent_t ev_gather_all = nullptr;
  bool gather_pending = false;

  // streams and events of the overlapped backward
  cudaStream_t s_dw = nullptr;    // weight-gradient GEMMs
  cudaStream_t s_comm = nullptr;  // data-parallel gradient all-reduce buckets
  std::vector<cudaEvent_t> ev_dgate, ev_rms2, ev_attn, ev_dw_done, ev_comm;
  cudaEvent_t ev_ce = nullptr, ev_de = nullptr, ev_main_done = nullptr, ev_comm_all = nullptr;
  bool overlap_allreduce = false;  // set by the train step of a data-parallel context
  bool layer_sumsq = false;        // set by the train step: grad-norm partials per final gradient segment

  // timing
  cudaEvent_t ev[8] = {};
  unsigned ev_recorded = 0;  // bit i: phase pair i (fwd, bwd, comm, opt) has been recorded
  bool profiling = false;
  std::vector<rt::KernelEvent> kevents;
  std::vector<cudaEvent_t> event_pool;
  size_t event_pool_used = 0;
  rt_timings acc{};
};
