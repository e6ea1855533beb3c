//! cuda-bridge: `extern "C"` binding of librustane_cuda.so, the B200 (sm_100a)
//! replacement of the `ane` crate surface the engine uses
//! (crates/ane-bridge/src/lib.rs:1-9; compile / eval at layer.rs:237-275, 600-602).
//!
//! Every function mirrors a declaration of include/rustane_cuda.h with the same
//! argument order and C types.  Status convention: 0 = OK, negative = error code
//! (RT_ERR_*); `check` turns a non-zero status into the panic the reference's
//! `.expect()` calls produce (layer.rs:243-259, 474).
//!
//! Not built in this repository's image: it has no Rust toolchain.  The header
//! is the source of truth; tests/test_cuda_bridge.py keeps this file in step.
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

pub const RT_OK: c_int = 0;
pub const RT_ERR_ARG: c_int = -1;
pub const RT_ERR_SHAPE: c_int = -2;
pub const RT_ERR_CUDA: c_int = -3;
pub const RT_ERR_OOM: c_int = -4;
pub const RT_ERR_TOKEN: c_int = -5;
pub const RT_ERR_DEVICE: c_int = -6;
pub const RT_ERR_NCCL: c_int = -7;
pub const RT_ERR_STATE: c_int = -8;
pub const RT_ERR_NONFINITE: c_int = -9;
pub const RT_CTX_TRAIN: c_int = 0;
pub const RT_CTX_FORWARD_ONLY: c_int = 1;
pub const RT_DIST_DATA_PARALLEL: c_int = 0;
pub const RT_DIST_TENSOR_PARALLEL: c_int = 1;

/// ModelConfig (crates/engine/src/model.rs:5-17).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct rt_model_config {
    pub dim: i32,
    pub hidden: i32,
    pub heads: i32,
    pub kv_heads: i32,
    pub hd: i32,
    pub seq: i32,
    pub nlayers: i32,
    pub vocab: i32,
    pub q_dim: i32,
    pub kv_dim: i32,
    pub gqa_ratio: i32,
}

/// TrainConfig (crates/engine/src/full_model.rs:34-70).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct rt_train_config {
    pub max_lr: f32,
    pub min_lr_frac: f32,
    pub warmup_steps: u32,
    pub total_steps: u32,
    pub beta1: f32,
    pub beta2: f32,
    pub eps: f32,
    pub weight_decay: f32,
    pub matrix_lr_scale: f32,
    pub embed_lr_scale: f32,
    pub loss_scale: f32,
    pub accum_steps: u32,
    pub grad_clip: f32,
    pub softcap: f32,
}

/// LayerWeights / LayerGrads / LayerOptState host pointers (layer.rs:16-39, training.rs:11-21).
#[repr(C)]
pub struct rt_layer_ptrs {
    pub wq: *mut f32,
    pub wk: *mut f32,
    pub wv: *mut f32,
    pub wo: *mut f32,
    pub w1: *mut f32,
    pub w3: *mut f32,
    pub w2: *mut f32,
    pub gamma1: *mut f32,
    pub gamma2: *mut f32,
}

/// ModelWeights / ModelGrads / ModelOptState host pointers (full_model.rs:13-31);
/// `layers` points to cfg.nlayers entries.
#[repr(C)]
pub struct rt_model_ptrs {
    pub embed: *mut f32,
    pub gamma_final: *mut f32,
    pub layers: *mut rt_layer_ptrs,
}

/// Device-side phase and kernel timings (CUDA events on the context stream).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct rt_timings {
    pub fwd_ms: f64,
    pub bwd_ms: f64,
    pub comm_ms: f64,
    pub opt_ms: f64,
    pub gemm_ms: f64,
    pub gemm_flops: f64,
    pub attn_ms: f64,
    pub attn_flops: f64,
    pub other_ms: f64,
    pub gemm_launches: i64,
    pub attn_launches: i64,
    pub other_launches: i64,
    pub kernel_launches: i64,
}

/// AdamConfig (crates/engine/src/cpu/adam.rs:12-30) for the single-layer step.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct rt_adam_config {
    pub lr: f32,
    pub beta1: f32,
    pub beta2: f32,
    pub eps: f32,
    pub weight_decay: f32,
}

/// Opaque context: device arenas, streams and (optionally) a communicator.
#[repr(C)]
pub struct rt_ctx {
    _p: [u8; 0],
}

/// Opaque memory-mapped u16 token file (data.rs:11-39).
#[repr(C)]
pub struct rt_tokens {
    _p: [u8; 0],
}

extern "C" {
    pub fn rt_ctx_create(cfg: *const rt_model_config, device: c_int, max_batch: c_int, flags: c_int, out: *mut *mut rt_ctx) -> c_int;
    pub fn rt_ctx_destroy(ctx: *mut rt_ctx) -> c_int;
    pub fn rt_last_error(ctx: *const rt_ctx) -> *const c_char;
    pub fn rt_ctx_device_bytes(ctx: *const rt_ctx, out: *mut i64) -> c_int;
    pub fn rt_weights_upload(ctx: *mut rt_ctx, w: *const rt_model_ptrs) -> c_int;
    pub fn rt_weights_download(ctx: *mut rt_ctx, w: *const rt_model_ptrs) -> c_int;
    pub fn rt_grads_download(ctx: *mut rt_ctx, g: *const rt_model_ptrs) -> c_int;
    pub fn rt_grads_upload(ctx: *mut rt_ctx, g: *const rt_model_ptrs) -> c_int;
    pub fn rt_opt_download(ctx: *mut rt_ctx, m: *const rt_model_ptrs, v: *const rt_model_ptrs) -> c_int;
    pub fn rt_opt_upload(ctx: *mut rt_ctx, m: *const rt_model_ptrs, v: *const rt_model_ptrs) -> c_int;
    pub fn rt_weights_init_normal(ctx: *mut rt_ctx, seed: u64, std: f32) -> c_int;
    pub fn rt_lcg_fill(out: *mut f32, n: i64, scale: f32) -> c_int;
    pub fn rt_forward(ctx: *mut rt_ctx, tokens: *const u32, targets: *const u32, batch: c_int, softcap: f32, loss_out: *mut f32, per_token_loss: *mut f32) -> c_int;
    pub fn rt_logits_download(ctx: *mut rt_ctx, logits: *mut f32) -> c_int;
    pub fn rt_backward(ctx: *mut rt_ctx, softcap: f32, loss_scale: f32) -> c_int;
    pub fn rt_grads_zero(ctx: *mut rt_ctx) -> c_int;
    pub fn rt_grad_norm(ctx: *mut rt_ctx, norm_out: *mut f32) -> c_int;
    pub fn rt_last_grad_norm(ctx: *mut rt_ctx, norm_out: *mut f32) -> c_int;
    pub fn rt_clip_grads(ctx: *mut rt_ctx, max_norm: f32) -> c_int;
    pub fn rt_update_weights(ctx: *mut rt_ctx, t: u32, lr: f32, tc: *const rt_train_config, grad_scale: f32) -> c_int;
    pub fn rt_learning_rate(step: u32, tc: *const rt_train_config) -> f32;
    pub fn rt_train_step(ctx: *mut rt_ctx, tokens: *const u32, targets: *const u32, batch: c_int, step: u32, tc: *const rt_train_config, loss_out: *mut f32) -> c_int;
    pub fn rt_stage_batch(ctx: *mut rt_ctx, slot: c_int, tokens: *const u32, targets: *const u32, batch: c_int) -> c_int;
    pub fn rt_train_step_staged(ctx: *mut rt_ctx, slot: c_int, step: u32, tc: *const rt_train_config, loss_out: *mut f32) -> c_int;
    pub fn rt_forward_staged(ctx: *mut rt_ctx, slot: c_int, softcap: f32) -> c_int;
    pub fn rt_sync(ctx: *mut rt_ctx, loss_out: *mut f32) -> c_int;
    pub fn rt_join(ctx: *mut rt_ctx) -> c_int;
    pub fn rt_ctx_stream(ctx: *const rt_ctx, stream_out: *mut *mut c_void) -> c_int;
    pub fn rt_last_h2d_bytes(ctx: *const rt_ctx, out: *mut i64) -> c_int;
    pub fn rt_layer_forward(ctx: *mut rt_ctx, layer: c_int, x: *const f32, batch: c_int, y: *mut f32) -> c_int;
    pub fn rt_layer_backward(ctx: *mut rt_ctx, layer: c_int, dy: *const f32, dx: *mut f32) -> c_int;
    pub fn rt_layer_train_step(ctx: *mut rt_ctx, layer: c_int, x: *const f32, batch: c_int, t: u32, cfg: *const rt_adam_config, loss_out: *mut f32) -> c_int;
    pub fn rt_tokens_open(path: *const c_char, out: *mut *mut rt_tokens) -> c_int;
    pub fn rt_tokens_close(t: *mut rt_tokens) -> c_int;
    pub fn rt_tokens_len(t: *const rt_tokens, n_out: *mut i64) -> c_int;
    pub fn rt_tokens_read(t: *const rt_tokens, start: i64, len: i64, out: *mut u32) -> c_int;
    pub fn rt_tokens_train_window(t: *const rt_tokens, step: u32, micro: u32, seq: c_int, tokens: *mut u32, targets: *mut u32) -> c_int;
    pub fn rt_tokens_val_window(t: *const rt_tokens, vs: u32, seq: c_int, tokens: *mut u32, targets: *mut u32) -> c_int;
    pub fn rt_compute_bpb(losses: *const f32, targets: *const u32, n: i64, token_bytes: *const i32, n_token_bytes: i32, bpb_out: *mut f32, nats_out: *mut f32, bytes_out: *mut i64) -> c_int;
    pub fn rt_checkpoint_write(path: *const c_char, cfg: *const rt_model_config, step: u32, w: *const rt_model_ptrs, m: *const rt_model_ptrs, v: *const rt_model_ptrs) -> c_int;
    pub fn rt_checkpoint_read(path: *const c_char, cfg: *const rt_model_config, step_out: *mut u32, version_out: *mut u32, w: *const rt_model_ptrs, m: *const rt_model_ptrs, v: *const rt_model_ptrs) -> c_int;
    pub fn rt_nccl_unique_id(out128: *mut u8) -> c_int;
    pub fn rt_tp_shard(heads: c_int, hidden: c_int, world: c_int, rank: c_int, head0: *mut c_int, heads_loc: *mut c_int, hid0: *mut c_int, hid_loc: *mut c_int) -> c_int;
    pub fn rt_dist_init(ctx: *mut rt_ctx, world: c_int, rank: c_int, unique_id128: *const u8, mode: c_int, timeout_ms: c_int) -> c_int;
    pub fn rt_dist_ranks(ctx: *const rt_ctx, nranks_out: *mut c_int) -> c_int;
    pub fn rt_grad_allreduce(ctx: *mut rt_ctx) -> c_int;
    pub fn rt_profile(ctx: *mut rt_ctx, enable: c_int) -> c_int;
    pub fn rt_get_timings(ctx: *mut rt_ctx, out: *mut rt_timings) -> c_int;
    pub fn rt_kernel_gemm(a: *const c_void, lda: i64, a_mn: c_int, b: *const c_void, ldb: i64, b_mn: c_int, M: c_int, N: c_int, K: c_int, epi: c_int, out: *mut c_void, ldo: i64, out2: *mut c_void, ldo2: i64, aux: *const c_void, ld_aux: i64, alpha: f32, beta: c_int, rope_cos: *const f32, rope_sin: *const f32, seq: c_int, rope_cols: c_int, n_half: c_int, force_bn: c_int, dev_err: *mut c_int, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_attention_fwd(qkv: *const c_void, out: *mut c_void, lse2: *mut f32, batch: c_int, seq: c_int, heads: c_int, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_attention_bwd(qkv: *const c_void, out: *const c_void, lse2: *const f32, dout: *const c_void, dvec: *mut f32, dqkv: *mut c_void, rope_cos_b: *const f32, rope_sin_b: *const f32, batch: c_int, seq: c_int, heads: c_int, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_attention_bwd_tc(qkv: *const c_void, out: *const c_void, lse2: *const f32, dout: *const c_void, dvec: *mut f32, ds_scratch: *mut c_void, dqkv: *mut c_void, rope_cos_b: *const f32, rope_sin_b: *const f32, batch: c_int, seq: c_int, heads: c_int, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_attention_bwd_scratch_bytes(batch: c_int, seq: c_int, heads: c_int) -> i64;
    pub fn rt_kernel_attention_bwd_noalloc(qkv: *const c_void, out: *const c_void, lse2: *const f32, dout: *const c_void, dqkv: *mut c_void, rope_cos_b: *const f32, rope_sin_b: *const f32, batch: c_int, seq: c_int, heads: c_int, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_rmsnorm_fwd(x: *const f32, gamma: *const f32, out_bf16: *mut c_void, rms_inv: *mut f32, M: c_int, D: c_int, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_rmsnorm_bwd(dy: *const f32, x: *const f32, gamma: *const f32, rms_inv: *const f32, resid: *const f32, dx: *mut f32, dx_bf16: *mut c_void, bf16_scale: f32, dgamma: *mut f32, accumulate: c_int, partials: *mut f32, M: c_int, D: c_int, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_rmsnorm_bwd_partials(M: c_int) -> c_int;
    pub fn rt_kernel_embed_gather(E: *const f32, tok: *const u32, x: *mut f32, M: c_int, D: c_int, V: c_int, dev_err: *mut c_int, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_embed_scatter(dx: *const f32, perm: *const i32, seg_start: *const i32, seg_tok: *const u32, nseg: c_int, dE: *mut f32, D: c_int, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_ce_fwd(logits: *const f32, tgt: *const u32, row_loss: *mut f32, row_lse: *mut f32, M: c_int, V: c_int, softcap: f32, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_ce_bwd(logits: *const f32, row_lse: *const f32, tgt: *const u32, dl_bf16: *mut c_void, M: c_int, V: c_int, softcap: f32, scale: f32, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_adam(param: *mut f32, grad: *const f32, m: *mut f32, v: *mut f32, param_bf16: *mut c_void, n: i64, t: u32, lr: f32, beta1: f32, beta2: f32, eps: f32, weight_decay: f32, grad_scale: f32, stream: *mut c_void) -> c_int;
    pub fn rt_kernel_l2norm(x: *const f32, n: i64, partials: *mut f32, out_norm: *mut f32, stream: *mut c_void) -> c_int;
}

/// Status -> the reference's `.expect()` behaviour: panic with the library's message.
pub fn check(ctx: *const rt_ctx, rc: c_int, what: &str) {
    if rc != RT_OK {
        let msg = unsafe { std::ffi::CStr::from_ptr(rt_last_error(ctx)) }.to_string_lossy();
        panic!("{what} failed ({rc}): {msg}");
    }
}

/// Owner of one `rt_ctx`: what `CompiledKernels::compile` (layer.rs:237-275) holds
/// in the engine.  Dropping it destroys the context (device memory, streams,
/// communicator).
pub struct Context {
    pub raw: *mut rt_ctx,
}

impl Context {
    pub fn new(cfg: &rt_model_config, device: i32, max_batch: i32, flags: c_int) -> Context {
        let mut raw: *mut rt_ctx = std::ptr::null_mut();
        let rc = unsafe { rt_ctx_create(cfg, device, max_batch, flags, &mut raw) };
        check(std::ptr::null(), rc, "rt_ctx_create");
        Context { raw }
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        if !self.raw.is_null() {
            unsafe { rt_ctx_destroy(self.raw) };
        }
    }
}
