"""ctypes binding of librustane_cuda.so (declared in include/rustane_cuda.h).

The library is the product; this module only loads it and declares argument
types.  It raises if the shared object is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

from .model import RtModelConfig
from .tensors import RtModelPtrs

LIB_PATH = Path(__file__).resolve().with_name("librustane_cuda.so")
HEADER = Path(__file__).resolve().parent.parent / "include" / "rustane_cuda.h"

RT_OK = 0
ERRORS = {
    -1: "RT_ERR_ARG", -2: "RT_ERR_SHAPE", -3: "RT_ERR_CUDA", -4: "RT_ERR_OOM", -5: "RT_ERR_TOKEN",
    -6: "RT_ERR_DEVICE", -7: "RT_ERR_NCCL", -8: "RT_ERR_STATE", -9: "RT_ERR_NONFINITE",
}
RT_ERR_ARG, RT_ERR_SHAPE, RT_ERR_CUDA, RT_ERR_OOM, RT_ERR_TOKEN, RT_ERR_DEVICE, RT_ERR_NCCL, RT_ERR_STATE, \
    RT_ERR_NONFINITE = range(-1, -10, -1)
RT_CTX_TRAIN, RT_CTX_FORWARD_ONLY = 0, 1
RT_DIST_DATA_PARALLEL, RT_DIST_TENSOR_PARALLEL = 0, 1

EPI_BF16, EPI_F32, EPI_F32_ACC, EPI_RESIDUAL, EPI_ROPE, EPI_SWIGLU, EPI_SWIGLU_BWD, EPI_BF16_ROWDOT = range(8)


class RtTrainConfig(ctypes.Structure):
    _fields_ = [("max_lr", ctypes.c_float), ("min_lr_frac", ctypes.c_float), ("warmup_steps", ctypes.c_uint32),
                ("total_steps", ctypes.c_uint32), ("beta1", ctypes.c_float), ("beta2", ctypes.c_float),
                ("eps", ctypes.c_float), ("weight_decay", ctypes.c_float), ("matrix_lr_scale", ctypes.c_float),
                ("embed_lr_scale", ctypes.c_float), ("loss_scale", ctypes.c_float),
                ("accum_steps", ctypes.c_uint32), ("grad_clip", ctypes.c_float), ("softcap", ctypes.c_float)]


class RtAdamConfig(ctypes.Structure):  # crates/engine/src/cpu/adam.rs:12-30
    _fields_ = [(n, ctypes.c_float) for n in ("lr", "beta1", "beta2", "eps", "weight_decay")]


class RtTimings(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in ("fwd_ms", "bwd_ms", "comm_ms", "opt_ms", "gemm_ms", "gemm_flops",
                                               "attn_ms", "attn_flops", "other_ms")] + \
               [(n, ctypes.c_int64) for n in ("gemm_launches", "attn_launches", "other_launches",
                                              "kernel_launches")]


c_int, c_int64, c_float, c_void_p, c_uint32 = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_uint32
c_float_p = ctypes.POINTER(ctypes.c_float)
c_uint32_p = ctypes.POINTER(ctypes.c_uint32)
c_uint8_p = ctypes.POINTER(ctypes.c_uint8)
P_CFG = ctypes.POINTER(RtModelConfig)
P_TC = ctypes.POINTER(RtTrainConfig)
P_PTRS = ctypes.POINTER(RtModelPtrs)

# name -> (restype, argtypes); must cover every function include/rustane_cuda.h declares
SIGNATURES: dict[str, tuple] = {
    "rt_ctx_create": (c_int, [P_CFG, c_int, c_int, c_int, ctypes.POINTER(c_void_p)]),
    "rt_ctx_destroy": (c_int, [c_void_p]),
    "rt_last_error": (ctypes.c_char_p, [c_void_p]),
    "rt_ctx_device_bytes": (c_int, [c_void_p, ctypes.POINTER(c_int64)]),
    "rt_weights_upload": (c_int, [c_void_p, P_PTRS]),
    "rt_weights_download": (c_int, [c_void_p, P_PTRS]),
    "rt_grads_download": (c_int, [c_void_p, P_PTRS]),
    "rt_grads_upload": (c_int, [c_void_p, P_PTRS]),
    "rt_opt_download": (c_int, [c_void_p, P_PTRS, P_PTRS]),
    "rt_opt_upload": (c_int, [c_void_p, P_PTRS, P_PTRS]),
    "rt_weights_init_normal": (c_int, [c_void_p, ctypes.c_uint64, c_float]),
    "rt_lcg_fill": (c_int, [c_float_p, c_int64, c_float]),
    "rt_forward": (c_int, [c_void_p, c_uint32_p, c_uint32_p, c_int, c_float, c_float_p, c_float_p]),
    "rt_logits_download": (c_int, [c_void_p, c_float_p]),
    "rt_backward": (c_int, [c_void_p, c_float, c_float]),
    "rt_grads_zero": (c_int, [c_void_p]),
    "rt_grad_norm": (c_int, [c_void_p, c_float_p]),
    "rt_last_grad_norm": (c_int, [c_void_p, c_float_p]),
    "rt_clip_grads": (c_int, [c_void_p, c_float]),
    "rt_update_weights": (c_int, [c_void_p, c_uint32, c_float, P_TC, c_float]),
    "rt_learning_rate": (c_float, [c_uint32, P_TC]),
    "rt_train_step": (c_int, [c_void_p, c_uint32_p, c_uint32_p, c_int, c_uint32, P_TC, c_float_p]),
    "rt_stage_batch": (c_int, [c_void_p, c_int, c_uint32_p, c_uint32_p, c_int]),
    "rt_train_step_staged": (c_int, [c_void_p, c_int, c_uint32, P_TC, c_float_p]),
    "rt_forward_staged": (c_int, [c_void_p, c_int, c_float]),
    "rt_sync": (c_int, [c_void_p, c_float_p]),
    "rt_ctx_stream": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "rt_last_h2d_bytes": (c_int, [c_void_p, ctypes.POINTER(c_int64)]),
    "rt_nccl_unique_id": (c_int, [c_uint8_p]),
    "rt_dist_init": (c_int, [c_void_p, c_int, c_int, c_uint8_p, c_int, c_int]),
    "rt_dist_ranks": (c_int, [c_void_p, ctypes.POINTER(c_int)]),
    "rt_tp_shard": (c_int, [c_int, c_int, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                            ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "rt_grad_allreduce": (c_int, [c_void_p]),
    "rt_join": (c_int, [c_void_p]),
    "rt_tokens_open": (c_int, [ctypes.c_char_p, ctypes.POINTER(c_void_p)]),
    "rt_tokens_close": (c_int, [c_void_p]),
    "rt_tokens_len": (c_int, [c_void_p, ctypes.POINTER(c_int64)]),
    "rt_tokens_read": (c_int, [c_void_p, c_int64, c_int64, c_uint32_p]),
    "rt_tokens_train_window": (c_int, [c_void_p, c_uint32, c_uint32, c_int, c_uint32_p, c_uint32_p]),
    "rt_tokens_val_window": (c_int, [c_void_p, c_uint32, c_int, c_uint32_p, c_uint32_p]),
    "rt_compute_bpb": (c_int, [c_float_p, c_uint32_p, c_int64, ctypes.POINTER(ctypes.c_int32), ctypes.c_int32,
                               c_float_p, c_float_p, ctypes.POINTER(c_int64)]),
    "rt_checkpoint_write": (c_int, [ctypes.c_char_p, P_CFG, c_uint32, ctypes.POINTER(RtModelPtrs),
                                    ctypes.POINTER(RtModelPtrs), ctypes.POINTER(RtModelPtrs)]),
    "rt_checkpoint_read": (c_int, [ctypes.c_char_p, P_CFG, ctypes.POINTER(c_uint32), ctypes.POINTER(c_uint32),
                                   ctypes.POINTER(RtModelPtrs), ctypes.POINTER(RtModelPtrs),
                                   ctypes.POINTER(RtModelPtrs)]),
    "rt_layer_forward": (c_int, [c_void_p, c_int, c_float_p, c_int, c_float_p]),
    "rt_layer_backward": (c_int, [c_void_p, c_int, c_float_p, c_float_p]),
    "rt_layer_train_step": (c_int, [c_void_p, c_int, c_float_p, c_int, c_uint32, ctypes.POINTER(RtAdamConfig),
                                    c_float_p]),
    "rt_profile": (c_int, [c_void_p, c_int]),
    "rt_get_timings": (c_int, [c_void_p, ctypes.POINTER(RtTimings)]),
    "rt_kernel_gemm": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int,
                               c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_float, c_int,
                               c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "rt_kernel_attention_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "rt_kernel_attention_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_int, c_int, c_int, c_void_p]),
    "rt_kernel_attention_bwd_tc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                           c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "rt_kernel_attention_bwd_scratch_bytes": (c_int64, [c_int, c_int, c_int]),
    "rt_kernel_attention_bwd_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                                c_void_p, c_int, c_int, c_int, c_void_p]),
    "rt_kernel_rmsnorm_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "rt_kernel_rmsnorm_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_float, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p]),
    "rt_kernel_rmsnorm_bwd_partials": (c_int, [c_int]),
    "rt_kernel_embed_gather": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "rt_kernel_embed_scatter": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p]),
    "rt_kernel_ce_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "rt_kernel_ce_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_float, c_void_p]),
    "rt_kernel_adam": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_uint32, c_float,
                               c_float, c_float, c_float, c_float, c_float, c_void_p]),
    "rt_kernel_l2norm": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
}

_lib = None


class RustaneError(RuntimeError):
    def __init__(self, code: int, msg: str = ""):
        self.code = code
        super().__init__(f"{ERRORS.get(code, code)}{': ' + msg if msg else ''}")


def lib() -> ctypes.CDLL:
    """Load librustane_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m rustane_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(code: int, ctx=None) -> None:
    if code != RT_OK:
        msg = lib().rt_last_error(ctx).decode(errors="replace") if (ctx is not None or code != RT_OK) else ""
        raise RustaneError(code, msg)
