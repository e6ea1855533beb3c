/*
 * rustane_cuda.h — C ABI of librustane_cuda.so, the B200 (sm_100a) engine for
 * rustane's language-model step: forward pass, backward pass and AdamW.
 *
 * This library is the `cuda-bridge` that replaces the `ane` crate surface the
 * engine crate binds today (crates/ane-bridge/src/lib.rs:1-9; graph build +
 * compile + eval at crates/engine/src/layer.rs:237-275, :600-602), the MIL
 * graph builders (the files of crates/engine/src/kernels/) and the Accelerate
 * CPU ops (crates/engine/src/cpu/).  Each entry point below names the reference
 * interface it replaces.
 *
 * Conventions
 *  - Every function returns an int status: RT_OK (0) or a negative RT_ERR_*.
 *    rt_last_error(ctx) returns a human-readable message for the last failure
 *    on that context (the reference panics via .expect(); the Rust binding maps
 *    non-zero status back to that panic).
 *  - Host pointers are borrowed for the duration of the call only.  Device
 *    memory is owned by the context.  Calls on one context are not thread-safe.
 *    Model-level calls are synchronous at return.
 *  - Host tensors use the reference layouts: row-major fp32, wq/wk/wv [dim,
 *    q_dim|kv_dim], wo [q_dim, dim], w1/w3/w2 [dim, hidden], embed [vocab, dim],
 *    gammas [dim].  Token ids are uint32 (the reference's u16 data files are
 *    widened by the caller, crates/engine/src/full_model.rs:683-684).
 *  - A batch is `batch` sequences of cfg.seq tokens each, processed in one
 *    pass; gradients are the SUM over sequences, exactly as the reference's
 *    gradient accumulation over `accum_steps` microbatches
 *    (full_model.rs:680-694), and the returned loss is the MEAN over sequences.
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

/* rt_ctx_create flags */
#define RT_CTX_TRAIN 0        /* fp32 master weights, grads, Adam moments, cached activations */
#define RT_CTX_FORWARD_ONLY 1 /* bf16 weights only, activations reused layer to layer        */

/* rt_dist_init modes */
#define RT_DIST_DATA_PARALLEL 0   /* gradients summed over ranks before grad-norm / AdamW (sharded AdamW) */
#define RT_DIST_TENSOR_PARALLEL 1 /* forward-only: heads / hidden sharded, all-reduce after Wo and W2 */

/* ----------------------------------------------------------------- types */

/* crates/engine/src/model.rs:5-17 (ModelConfig). */
typedef struct rt_model_config {
  int32_t dim, hidden, heads, kv_heads, hd, seq, nlayers, vocab, q_dim, kv_dim, gqa_ratio;
} rt_model_config;

/* crates/engine/src/full_model.rs:34-70 (TrainConfig). */
typedef struct rt_train_config {
  float max_lr, min_lr_frac;
  uint32_t warmup_steps, total_steps;
  float beta1, beta2, eps, weight_decay, matrix_lr_scale, embed_lr_scale, loss_scale;
  uint32_t accum_steps;
  float grad_clip, softcap;
} rt_train_config;

/* Per-layer host tensors (crates/engine/src/layer.rs:16-39 LayerWeights /
 * LayerGrads; training.rs:11-21 LayerOptState uses the same shapes). */
typedef struct rt_layer_ptrs {
  float *wq, *wk, *wv, *wo, *w1, *w3, *w2, *gamma1, *gamma2;
} rt_layer_ptrs;

/* Whole-model host tensors (full_model.rs:13-31 ModelWeights / ModelGrads /
 * ModelOptState); `layers` points to cfg.nlayers entries. */
typedef struct rt_model_ptrs {
  float* embed;
  float* gamma_final;
  rt_layer_ptrs* layers;
} rt_model_ptrs;

/* Device-side phase and kernel timings (CUDA events on the context stream). */
typedef struct rt_timings {
  double fwd_ms, bwd_ms, comm_ms, opt_ms; /* last forward / backward / all-reduce span / norm+AdamW */
  double gemm_ms, gemm_flops;             /* accumulated over GEMM launches while profiling   */
  double attn_ms, attn_flops;             /* accumulated over attention launches              */
  double other_ms;                        /* accumulated over all other kernels               */
  int64_t gemm_launches, attn_launches, other_launches;
  int64_t kernel_launches; /* every kernel this context launched since creation */
} rt_timings;

/* crates/engine/src/cpu/adam.rs:12-30 (AdamConfig) for the single-layer step. */
typedef struct rt_adam_config {
  float lr, beta1, beta2, eps, weight_decay;
} rt_adam_config;

typedef struct rt_ctx rt_ctx;

/* --------------------------------------------------------- context / data */

/* Allocate a context on `device` for batches of up to `max_batch` sequences.
 * Replaces CompiledKernels::compile (crates/engine/src/layer.rs:237-275) plus
 * the workspaces ModelForwardWorkspace / ModelBackwardWorkspace
 * (full_model.rs:123-185). */
RT_API int rt_ctx_create(const rt_model_config* cfg, int device, int max_batch, int flags, rt_ctx** out);
RT_API int rt_ctx_destroy(rt_ctx* ctx);
RT_API const char* rt_last_error(const rt_ctx* ctx);
/* Bytes of device memory the context holds. */
RT_API int rt_ctx_device_bytes(const rt_ctx* ctx, int64_t* out);

/* Copy weights host -> device (fp32 master + bf16 compute copy). */
RT_API int rt_weights_upload(rt_ctx* ctx, const rt_model_ptrs* w);
/* Copy weights device -> host (fp32 master; training contexts only). */
RT_API int rt_weights_download(rt_ctx* ctx, const rt_model_ptrs* w);
/* Gradients device <-> host (reference layout, ModelGrads). */
RT_API int rt_grads_download(rt_ctx* ctx, const rt_model_ptrs* g);
RT_API int rt_grads_upload(rt_ctx* ctx, const rt_model_ptrs* g);
/* Adam moments device <-> host (ModelOptState). */
RT_API int rt_opt_download(rt_ctx* ctx, const rt_model_ptrs* m, const rt_model_ptrs* v);
RT_API int rt_opt_upload(rt_ctx* ctx, const rt_model_ptrs* m, const rt_model_ptrs* v);
/* Device-side init: every matrix and the embedding N(0, std) from a counter-based
 * stream keyed by `seed`, gammas = 1, moments and gradients 0.  Used for the
 * configurations whose fp32 weights do not fit comfortably in host memory. */
RT_API int rt_weights_init_normal(rt_ctx* ctx, uint64_t seed, float std);

/* Host-side helper: the reference's LCG init stream (random_vec,
 * crates/engine/src/layer.rs:404-413): seed = 42 + n. */
RT_API int rt_lcg_fill(float* out, int64_t n, float scale);

/* ---------------------------------------------------------- model step */

/* Forward of `batch` sequences + cross-entropy (full_model::forward_ws,
 * full_model.rs:187-247; per_token_loss = forward_losses, :717-767).
 * tokens / targets: batch * seq uint32 ids.  loss_out: mean loss.
 * per_token_loss (nullable): batch * seq CE values.  Keeps the activations
 * for rt_backward (training contexts). */
RT_API int rt_forward(rt_ctx* ctx, const uint32_t* tokens, const uint32_t* targets, int batch, float softcap,
                      float* loss_out, float* per_token_loss);
/* Copy the last forward's logits (after softcap) to host, [batch*seq, vocab] fp32. */
RT_API int rt_logits_download(rt_ctx* ctx, float* logits);
/* Backward of the last forward (full_model::backward_ws, full_model.rs:250-331):
 * dlogits * loss_scale, gradients accumulate into the device grads. */
RT_API int rt_backward(rt_ctx* ctx, float softcap, float loss_scale);
/* ModelGrads::zero_out (full_model.rs:100-107). */
RT_API int rt_grads_zero(rt_ctx* ctx);
/* Global L2 norm of all gradients (grad_norm, full_model.rs:598-624). */
RT_API int rt_grad_norm(rt_ctx* ctx, float* norm_out);
/* The raw global gradient norm the last rt_train_step / rt_train_step_staged
 * (or rt_grad_norm) computed on the device, without recomputing it: the value
 * the training loop logs as gnorm / (accum * loss_scale) (bin/train.rs:252-290
 * calls grad_norm, full_model.rs:598-624, after each step).  Under data
 * parallelism it is the norm of the gradients summed over the ranks, so a
 * sharded step needs no gather to report it.  RT_ERR_STATE when no norm was
 * computed since the context was created or a single-layer call reused the
 * slot. */
RT_API int rt_last_grad_norm(rt_ctx* ctx, float* norm_out);
/* clip_grads (full_model.rs:627-645). */
RT_API int rt_clip_grads(rt_ctx* ctx, float max_norm);
/* AdamW with the reference's learning-rate groups (update_weights,
 * full_model.rs:490-593): embed lr*embed_lr_scale wd 0, gamma_final lr wd 0,
 * matrices lr*matrix_lr_scale wd weight_decay, gamma1/2 lr wd 0; t is 1-based. */
RT_API int rt_update_weights(rt_ctx* ctx, uint32_t t, float lr, const rt_train_config* tc, float grad_scale);
/* learning_rate (full_model.rs:334-342). */
RT_API float rt_learning_rate(uint32_t step, const rt_train_config* tc);
/* One optimizer step over `batch` sequences (train_step, full_model.rs:661-714,
 * with accum_steps = batch * world): zero grads, forward, backward with
 * tc->loss_scale, [data-parallel all-reduce], grad norm, clip rule, lr(step),
 * AdamW(t = step + 1).  The clip decision runs on the device (no host sync
 * inside the step).  loss_out: mean loss of this rank's sequences. */
RT_API int rt_train_step(rt_ctx* ctx, const uint32_t* tokens, const uint32_t* targets, int batch, uint32_t step,
                         const rt_train_config* tc, float* loss_out);

/* Device-resident inputs: upload a batch (tokens, targets and the embedding
 * scatter segments) into slot `slot` ahead of time, then run steps on it with
 * no host transfer.  rt_train_step_staged with loss_out == NULL returns
 * without waiting (asynchronous); rt_sync waits, checks the device error word
 * and optionally reads the last loss.  These are the train_step / forward_ws
 * of full_model.rs with the input copy hoisted out of the step. */
RT_API int rt_stage_batch(rt_ctx* ctx, int slot, const uint32_t* tokens, const uint32_t* targets, int batch);
RT_API int rt_train_step_staged(rt_ctx* ctx, int slot, uint32_t step, const rt_train_config* tc, float* loss_out);
RT_API int rt_forward_staged(rt_ctx* ctx, int slot, float softcap);
RT_API int rt_sync(rt_ctx* ctx, float* loss_out);
/* Make the context stream wait for work the last step left on the context's
 * other streams (the weight all-gathers of a sharded data-parallel step, which
 * the next forward otherwise waits for layer by layer).  Asynchronous: an event
 * recorded on the context stream after it covers the whole step. */
RT_API int rt_join(rt_ctx* ctx);
/* The context's CUDA stream (cudaStream_t) — every kernel of the context runs on it. */
RT_API int rt_ctx_stream(const rt_ctx* ctx, void** stream_out);
/* Bytes the last host-token call copied host -> device. */
RT_API int rt_last_h2d_bytes(const rt_ctx* ctx, int64_t* out);

/* ------------------------------------------------------- single layer
 * One transformer layer of a training context on its own (the engine's layer
 * API and the Phase-3 training loop).  Activations use the reference layout:
 * per sequence channel-first [dim][seq] fp32, `batch` sequences back to back.
 * The layer's weights are layer `layer` of the context's weights. */

/* layer::forward (layer.rs:443-...): y = the layer output; keeps the layer's
 * activations for rt_layer_backward (and invalidates the last model forward). */
RT_API int rt_layer_forward(rt_ctx* ctx, int layer, const float* x, int batch, float* y);
/* layer::backward (layer.rs:1355-1858) of the last rt_layer_forward of `layer`:
 * dx = gradient at the layer input; the layer's weight gradients accumulate
 * into the device grads (LayerGrads semantics). */
RT_API int rt_layer_backward(rt_ctx* ctx, int layer, const float* dy, float* dx);
/* training::train_step (training.rs:61-97): forward, loss = mean(y^2) (MSE
 * against zero), the layer's gradients zeroed then dy = 2 y / n backward,
 * and training::update_weights (training.rs:41-59): AdamW (adam::step,
 * cpu/adam.rs:37-85) with one config for all nine tensors, t 1-based. */
RT_API int rt_layer_train_step(rt_ctx* ctx, int layer, const float* x, int batch, uint32_t t,
                               const rt_adam_config* cfg, float* loss_out);

/* ------------------------------------------------------- host I/O
 * The engine's training-data and checkpoint files, host side only (no device). */

/* TokenData (crates/engine/src/data.rs:11-39): a memory-mapped file of
 * little-endian uint16 token ids. */
typedef struct rt_tokens rt_tokens;
RT_API int rt_tokens_open(const char* path, rt_tokens** out);
RT_API int rt_tokens_close(rt_tokens* t);
RT_API int rt_tokens_len(const rt_tokens* t, int64_t* n_out);
/* Tokens [start, start + len) widened to uint32. */
RT_API int rt_tokens_read(const rt_tokens* t, int64_t start, int64_t len, uint32_t* out);
/* Training window of microbatch `micro` at `step` (bin/train.rs:285-290,
 * data.rs:92-95): pos = (step*7919 + micro*104729) mod (n - seq - 1);
 * tokens = data[pos, pos+seq), targets = data[pos+1, pos+seq+1). */
RT_API int rt_tokens_train_window(const rt_tokens* t, uint32_t step, uint32_t micro, int seq, uint32_t* tokens,
                                  uint32_t* targets);
/* Validation window `vs` (bin/train.rs:128-131): pos = (vs*seq) mod (n - seq - 1). */
RT_API int rt_tokens_val_window(const rt_tokens* t, uint32_t vs, int seq, uint32_t* tokens, uint32_t* targets);
/* compute_bpb (data.rs:67-89) over n per-token losses (nats) and their target
 * ids, with the token_bytes.bin table (int32 byte length per id). */
RT_API int rt_compute_bpb(const float* losses, const uint32_t* targets, int64_t n, const int32_t* token_bytes,
                          int32_t n_token_bytes, float* bpb_out, float* nats_out, int64_t* bytes_out);
/* RSTK checkpoint (save_checkpoint, bin/train.rs:165-202): version 1 (m = v =
 * NULL) is the reference's file byte for byte; version 2 appends the AdamW
 * moments m and v, which the reference does not save.  The reader takes
 * either version, checks dim / nlayers / vocab / seq against cfg, and fills m
 * and v when the file has them and they are given. */
RT_API int rt_checkpoint_write(const char* path, const rt_model_config* cfg, uint32_t step, const rt_model_ptrs* w,
                               const rt_model_ptrs* m, const rt_model_ptrs* v);
RT_API int rt_checkpoint_read(const char* path, const rt_model_config* cfg, uint32_t* step_out,
                              uint32_t* version_out, const rt_model_ptrs* w, const rt_model_ptrs* m,
                              const rt_model_ptrs* v);

/* ------------------------------------------------------- multi-GPU */

/* NCCL unique id (128 bytes) for rank 0 to broadcast to the other ranks. */
RT_API int rt_nccl_unique_id(uint8_t* out128);
/* The tensor-parallel partition rt_dist_init applies (host only, no device):
 * rank `rank` of `world` owns heads [head0, head0 + heads_loc) and hidden
 * columns [hid0, hid0 + hid_loc).  The first heads % world ranks take one
 * extra head; the hidden columns are split likewise in 64-column units (52
 * heads over 8 ranks: 7,7,7,7,6,6,6,6).  Replaces the all-heads layout of
 * layer::forward_into (layer.rs:552-680), which has no sharded form. */
RT_API int rt_tp_shard(int heads, int hidden, int world, int rank, int* head0, int* heads_loc, int* hid0,
                       int* hid_loc);
/* Join a communicator of `world` ranks (one process per GPU).  mode:
 * RT_DIST_DATA_PARALLEL or RT_DIST_TENSOR_PARALLEL.  Collectives that do not
 * finish within timeout_ms abort the communicator and return RT_ERR_NCCL.
 * Data parallel: rt_train_step reduce-scatters each gradient segment (the
 * embedding, each layer's matrices, the gammas) as soon as the backward has
 * finished it, every rank runs AdamW on its 1/world chunk of every segment
 * (the grad norm is summed over the ranks first), and the weights the forward
 * reads are all-gathered -- the same update as an all-reduce of the gradients
 * followed by AdamW on every rank.  The fp32 matrices, the AdamW moments and the
 * gradients then stay sharded; rt_weights_download, rt_opt_download,
 * rt_grads_download, rt_grad_norm, rt_clip_grads, rt_update_weights and an
 * accumulating rt_backward gather them first, so every rank must make those
 * calls together.  When a segment does not split into 16-byte chunks per rank
 * (or RUSTANE_DP_ALLREDUCE=1 is set), the gradients are all-reduced instead.
 * A context joins one communicator: after a join with world > 1, a further
 * call returns RT_ERR_STATE.  A failed join (RT_ERR_NCCL) leaves the context
 * unchanged. */
RT_API int rt_dist_init(rt_ctx* ctx, int world, int rank, const uint8_t* unique_id128, int mode, int timeout_ms);
/* Ranks of the context's NCCL communicator as NCCL itself reports them
 * (ncclCommCount); 1 without a communicator.  No reference counterpart: the
 * reference runs on one device. */
RT_API int rt_dist_ranks(const rt_ctx* ctx, int* nranks_out);
/* Sum the gradients over the data-parallel ranks (one in-place all-reduce). */
RT_API int rt_grad_allreduce(rt_ctx* ctx);

/* ------------------------------------------------------- diagnostics */

/* Enable (1) / disable (0) per-kernel CUDA-event timing; resets the accumulators. */
RT_API int rt_profile(rt_ctx* ctx, int enable);
RT_API int rt_get_timings(rt_ctx* ctx, rt_timings* out);

/* -------------------------------------------------- kernel-level entries */

/* GEMM epilogue selector for rt_kernel_gemm. */
#define RT_EPI_BF16 0
#define RT_EPI_F32 1
#define RT_EPI_F32_ACC 2
#define RT_EPI_RESIDUAL 3
#define RT_EPI_ROPE 4
#define RT_EPI_SWIGLU 5
#define RT_EPI_SWIGLU_BWD 6
/* out = bf16(C) and out2 (fp32) [M/seq][N/128][seq] = per 128-column head, the
 * sum of bf16(C) * aux (bf16 [M][ld_aux]) over the head's columns: the rowsum
 * dO . O of the attention backward (sdpaBwd1, kernels/sdpa_bwd.rs:44-100) from
 * the GEMM that produces dO.  K-major A and B, N % 128 == 0, M % seq == 0;
 * 256-wide tiles (force_bn 0, 256 or -256). */
#define RT_EPI_BF16_ROWDOT 7

/* tcgen05 GEMM C[M,N] = sum_k A[m,k] B[n,k] (bf16 in, fp32 accumulate) with a
 * fused epilogue.  a_mn/b_mn select MN-major storage ([K][M] / [K][N]).
 * Replaces the DynMatmul / DualDynMatmul ANE graphs
 * (crates/engine/src/kernels/dyn_matmul.rs:15-86), the matmuls inside
 * sdpaFwd/ffnFused (kernels/sdpa_fwd.rs:80-83, kernels/ffn_fused.rs:48-72) and
 * the cblas_sgemm calls (crates/engine/src/cpu/vdsp.rs:128-136, :287-321).
 * force_bn: 0 lets the library choose; 128/192/256 force the single-CTA kernel
 * with that output tile width; -256/-128 force the CTA-pair kernel (a cluster
 * of two SMs owns a 256 x 256 / 256 x 192 / 256 x 128 tile; 192 needs K-major B,
 * else RT_ERR_SHAPE). */
RT_API int rt_kernel_gemm(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, int M, int N,
                          int K, int epi, void* out, int64_t ldo, void* out2, int64_t ldo2, const void* aux,
                          int64_t ld_aux, float alpha, int beta, const float* rope_cos, const float* rope_sin,
                          int seq, int rope_cols, int n_half, int force_bn, int* dev_err, void* stream);

/* Causal attention forward over qkv [batch*seq, 3*dim] bf16 (roped Q, K; V):
 * out [batch*seq, dim] bf16, lse2 [batch, heads, seq] fp32 (log2 domain).
 * Replaces the attention half of sdpaFwd (kernels/sdpa_fwd.rs:130-150). */
RT_API int rt_kernel_attention_fwd(const void* qkv, void* out, float* lse2, int batch, int seq, int heads,
                                   void* stream);
/* Causal attention backward: dqkv [batch*seq, 3*dim] bf16 with the RoPE backward
 * rotation applied to dQ and dK (rope tables [hd/2][seq], layer.rs:197-217).
 * dvec: scratch [batch, heads, seq] fp32.  Replaces sdpaBwd1 + sdpaBwd2
 * (kernels/sdpa_bwd.rs:44-162) and rope_backward_inplace (layer.rs:1880-1897). */
RT_API int rt_kernel_attention_bwd(const void* qkv, const void* out, const float* lse2, const void* dout,
                                   float* dvec, void* dqkv, const float* rope_cos_b, const float* rope_sin_b,
                                   int batch, int seq, int heads, void* stream);

/* The same backward on the tcgen05 tensor cores (what the model step runs):
 * dK / dV per 128-key block with S^T, dP^T, dV, dK in TMEM, then dQ from the
 * bf16 dS tiles kept in `ds_scratch`
 * (rt_kernel_attention_bwd_scratch_bytes(batch, seq, heads) bytes of device
 * memory).  lse2, dvec, ds_scratch and dqkv 16-byte aligned.  Deterministic:
 * every dQ element is summed in a fixed order (no atomics). */
RT_API int rt_kernel_attention_bwd_tc(const void* qkv, const void* out, const float* lse2, const void* dout,
                                      float* dvec, void* ds_scratch, void* dqkv, const float* rope_cos_b,
                                      const float* rope_sin_b, int batch, int seq, int heads, void* stream);
RT_API int64_t rt_kernel_attention_bwd_scratch_bytes(int batch, int seq, int heads);

/* Allocation-free variant of rt_kernel_attention_bwd, for callers that cannot
 * call cudaMalloc when they run the backward pass (device memory owned by
 * another allocator, or a loop that must not take cudaMalloc's implicit device
 * synchronisation).  No counterpart in the reference: it has no GPU path.  The
 * rowsum(dO * O) scratch comes from a 2 MiB array compiled into the library
 * (held by every GPU that loads it until exit) instead of the caller:
 * batch * heads * seq must be <= 524288, otherwise RT_ERR_SHAPE.  The first call
 * on a device looks up that array's device address (make it before any stream
 * capture).  All calls share the array: calls that overlap on the GPU race, so
 * order them on one stream.  Inputs and outputs as rt_kernel_attention_bwd. */
RT_API int rt_kernel_attention_bwd_noalloc(const void* qkv, const void* out, const float* lse2, const void* dout,
                                           void* dqkv, const float* rope_cos_b, const float* rope_sin_b, int batch,
                                           int seq, int heads, void* stream);

/* Row RMSNorm over x [M, D] fp32 -> out bf16, rms_inv [M]
 * (cpu/rmsnorm.rs:149-183, token-major). */
RT_API int rt_kernel_rmsnorm_fwd(const float* x, const float* gamma, void* out_bf16, float* rms_inv, int M, int D,
                                 void* stream);
/* RMSNorm backward (cpu/rmsnorm.rs:190-238, token-major): dx = ... + resid,
 * optional dx_bf16 = bf16(scale * dx); dgamma (accumulate ? += : =).
 * partials: scratch of rt_kernel_rmsnorm_bwd_partials(M) * D floats. */
RT_API int rt_kernel_rmsnorm_bwd(const float* dy, const float* x, const float* gamma, const float* rms_inv,
                                 const float* resid, float* dx, void* dx_bf16, float bf16_scale, float* dgamma,
                                 int accumulate, float* partials, int M, int D, void* stream);
RT_API int rt_kernel_rmsnorm_bwd_partials(int M);
/* Embedding gather (cpu/embedding.rs:8-16): x[m,:] = E[tok[m],:] exactly. */
RT_API int rt_kernel_embed_gather(const float* E, const uint32_t* tok, float* x, int M, int D, int V, int* dev_err,
                                  void* stream);
/* Embedding scatter-add (cpu/embedding.rs:34-44), deterministic: segments of
 * positions grouped by token (perm, seg_start[nseg+1], seg_tok[nseg]). */
RT_API int rt_kernel_embed_scatter(const float* dx, const int32_t* perm, const int32_t* seg_start,
                                   const uint32_t* seg_tok, int nseg, float* dE, int D, void* stream);
/* Cross-entropy forward / backward over fp32 logits rows (cpu/cross_entropy.rs:58-96,
 * softcap full_model.rs:232-239, 265-276). */
RT_API int rt_kernel_ce_fwd(const float* logits, const uint32_t* tgt, float* row_loss, float* row_lse, int M, int V,
                            float softcap, void* stream);
RT_API int rt_kernel_ce_bwd(const float* logits, const float* row_lse, const uint32_t* tgt, void* dl_bf16, int M,
                            int V, float softcap, float scale, void* stream);
/* Multi-tensor AdamW over one contiguous fp32 range (cpu/adam.rs:95-132),
 * optional bf16 copy of the updated parameters. */
RT_API int rt_kernel_adam(float* param, const float* grad, float* m, float* v, void* param_bf16, int64_t n,
                          uint32_t t, float lr, float beta1, float beta2, float eps, float weight_decay,
                          float grad_scale, void* stream);
/* Deterministic global L2 norm; partials: scratch of 1024 floats. */
RT_API int rt_kernel_l2norm(const float* x, int64_t n, float* partials, float* out_norm, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RUSTANE_CUDA_H */
