"""ctypes wrapper of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py to check or time the reference algorithm.  The
product (rustane_b200) never imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

from rustane_b200.model import ModelConfig, RtModelConfig
from rustane_b200.tensors import LayerTensors, ModelOptState, ModelTensors, RtLayerPtrs, RtModelPtrs

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"


class OrTrainConfig(ctypes.Structure):
    _fields_ = [("max_lr", ctypes.c_float), ("min_lr_frac", ctypes.c_float), ("warmup_steps", ctypes.c_uint32),
                ("total_steps", ctypes.c_uint32), ("beta1", ctypes.c_float), ("beta2", ctypes.c_float),
                ("eps", ctypes.c_float), ("weight_decay", ctypes.c_float), ("matrix_lr_scale", ctypes.c_float),
                ("embed_lr_scale", ctypes.c_float), ("loss_scale", ctypes.c_float),
                ("accum_steps", ctypes.c_uint32), ("grad_clip", ctypes.c_float), ("softcap", ctypes.c_float)]


def default_train_config(**kw) -> OrTrainConfig:
    """TrainConfig::default (crates/engine/src/full_model.rs:51-70)."""
    d = dict(max_lr=3e-4, min_lr_frac=0.1, warmup_steps=100, total_steps=10000, beta1=0.9, beta2=0.95, eps=1e-8,
             weight_decay=0.1, matrix_lr_scale=0.05, embed_lr_scale=5.0, loss_scale=256.0, accum_steps=10,
             grad_clip=1.0, softcap=0.0)
    d.update(kw)
    return OrTrainConfig(**d)


_lib = None
F = ctypes.POINTER(ctypes.c_float)
U32 = ctypes.POINTER(ctypes.c_uint32)


def numpy_blas_path() -> str | None:
    libs = Path(np.__file__).resolve().parent.parent / "numpy.libs"
    for p in sorted(libs.glob("libscipy_openblas64_*.so")):
        return str(p)
    return None


def build() -> Path:
    if not LIB.exists() or LIB.stat().st_mtime < (HERE / "oracle.cpp").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib(threads: int | None = None) -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        h = ctypes.CDLL(str(LIB))
        sig = {
            "or_init": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int]),
            "or_blas_name": (ctypes.c_char_p, []),
            "or_threads": (ctypes.c_int, []),
            "or_sgemm": (None, [ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                ctypes.c_float, F, ctypes.c_int64, F, ctypes.c_int64, ctypes.c_float, F,
                                ctypes.c_int64]),
            "or_random_vec": (None, [F, ctypes.c_int64, ctypes.c_float]),
            "or_rmsnorm_forward": (ctypes.c_float, [F, F, F, ctypes.c_int]),
            "or_rmsnorm_backward": (None, [F, F, F, ctypes.c_float, F, F, ctypes.c_int]),
            "or_rmsnorm_forward_cf": (None, [F, F, F, F, ctypes.c_int, ctypes.c_int]),
            "or_rmsnorm_backward_cf": (None, [F, F, F, F, F, F, ctypes.c_int, ctypes.c_int]),
            "or_ce_forward": (ctypes.c_float, [F, ctypes.c_int, ctypes.c_int, F]),
            "or_ce_backward": (None, [F, ctypes.c_int, ctypes.c_int, F]),
            "or_ce_forward_backward_batch": (ctypes.c_float, [F, U32, ctypes.c_int, ctypes.c_int, F, ctypes.c_float]),
            "or_adam_step": (None, [F, F, F, F, ctypes.c_int64, ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                                    ctypes.c_float, ctypes.c_float, ctypes.c_float]),
            "or_adam_step_fused": (None, [F, F, F, F, ctypes.c_int64, ctypes.c_uint32, ctypes.c_float,
                                          ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                          ctypes.c_float]),
            "or_embedding_forward": (None, [F, ctypes.c_int, U32, ctypes.c_int, F]),
            "or_embedding_backward": (None, [F, ctypes.c_int, U32, ctypes.c_int, F]),
            "or_embedding_backward_cf": (None, [F, ctypes.c_int, U32, ctypes.c_int, F]),
            "or_silu_forward": (None, [F, F, ctypes.c_int64]),
            "or_silu_backward": (None, [F, F, F, ctypes.c_int64]),
            "or_ws_create": (ctypes.c_void_p, [ctypes.POINTER(RtModelConfig), ctypes.c_int]),
            "or_ws_destroy": (None, [ctypes.c_void_p]),
            "or_rope_tables": (None, [ctypes.c_void_p, F, F, F, F]),
            "or_forward": (ctypes.c_int, [ctypes.POINTER(RtModelConfig), ctypes.POINTER(RtModelPtrs), U32, U32,
                                          ctypes.c_int, ctypes.c_float, ctypes.c_void_p, F, F, F]),
            "or_backward": (ctypes.c_int, [ctypes.POINTER(RtModelConfig), ctypes.POINTER(RtModelPtrs),
                                           ctypes.c_void_p, U32, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                           ctypes.POINTER(RtModelPtrs)]),
            "or_grad_norm": (ctypes.c_float, [ctypes.POINTER(RtModelConfig), ctypes.POINTER(RtModelPtrs)]),
            "or_clip_grads": (None, [ctypes.POINTER(RtModelConfig), ctypes.POINTER(RtModelPtrs), ctypes.c_float]),
            "or_learning_rate": (ctypes.c_float, [ctypes.c_uint32, ctypes.POINTER(OrTrainConfig)]),
            "or_update_weights": (None, [ctypes.POINTER(RtModelConfig), ctypes.POINTER(RtModelPtrs),
                                         ctypes.POINTER(RtModelPtrs), ctypes.POINTER(RtModelPtrs),
                                         ctypes.POINTER(RtModelPtrs), ctypes.c_uint32, ctypes.c_float,
                                         ctypes.POINTER(OrTrainConfig), ctypes.c_float]),
            "or_grads_zero": (None, [ctypes.POINTER(RtModelConfig), ctypes.POINTER(RtModelPtrs)]),
            "or_train_step_batch": (ctypes.c_float, [ctypes.POINTER(RtModelConfig), ctypes.POINTER(RtModelPtrs),
                                                     ctypes.POINTER(RtModelPtrs), ctypes.POINTER(RtModelPtrs),
                                                     ctypes.POINTER(RtModelPtrs), U32, U32, ctypes.c_int,
                                                     ctypes.c_uint32, ctypes.POINTER(OrTrainConfig),
                                                     ctypes.c_void_p, F]),
            "or_train_positions": (None, [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int64, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_int64)]),
            "or_layer_forward": (None, [ctypes.POINTER(RtModelConfig), ctypes.c_void_p, ctypes.POINTER(RtLayerPtrs),
                                        F, F]),
            "or_layer_backward": (None, [ctypes.POINTER(RtModelConfig), ctypes.c_void_p,
                                         ctypes.POINTER(RtLayerPtrs), F, ctypes.POINTER(RtLayerPtrs), F]),
            "or_layer_train_step": (ctypes.c_float, [ctypes.POINTER(RtModelConfig), ctypes.c_void_p,
                                                     ctypes.POINTER(RtLayerPtrs), ctypes.POINTER(RtLayerPtrs),
                                                     ctypes.POINTER(RtLayerPtrs), ctypes.POINTER(RtLayerPtrs), F,
                                                     ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                                                     ctypes.c_float, ctypes.c_float, ctypes.c_float]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        blas = numpy_blas_path()
        rc = h.or_init(blas.encode() if blas else None, int(threads or os.cpu_count() or 1))
        if rc != 0:
            h.or_init(None, int(threads or os.cpu_count() or 1))
        _lib = h
    return _lib


def fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(F)


def up(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(U32)


# ------------------------------------------------------------------ init
def random_vec(n: int, scale: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_random_vec(fp(out), n, scale)
    return out


def reference_init(cfg: ModelConfig) -> ModelTensors:
    """ModelWeights::random (full_model.rs:84-90; layer.rs:358-373): LCG seeded 42 + n,
    qkv scale 1/sqrt(dim), w1/w3 1/sqrt(hidden), wo = w2 = 0, embed 0.005, gammas 1."""
    t = ModelTensors.zeros(cfg)
    D, H = cfg.dim, cfg.hidden
    sq, sf = 1.0 / np.sqrt(np.float32(D)), 1.0 / np.sqrt(np.float32(H))
    qkv = {"wq": random_vec(D * cfg.q_dim, sq), "wk": random_vec(D * cfg.kv_dim, sq),
           "wv": random_vec(D * cfg.kv_dim, sq)}
    w1 = random_vec(D * H, sf)
    for L in t.layers:  # every layer gets the same values (seed depends only on n)
        L.wq[...] = qkv["wq"].reshape(L.wq.shape)
        L.wk[...] = qkv["wk"].reshape(L.wk.shape)
        L.wv[...] = qkv["wv"].reshape(L.wv.shape)
        L.w1[...] = w1.reshape(L.w1.shape)
        L.w3[...] = w1.reshape(L.w3.shape)
        L.gamma1[...] = 1.0
        L.gamma2[...] = 1.0
    t.embed[...] = random_vec(cfg.vocab * D, 0.005).reshape(t.embed.shape)
    t.gamma_final[...] = 1.0
    return t


def pattern_tokens(cfg: ModelConfig, batch: int = 1):
    """Tokens (i*31+7) % vocab and next-token targets (tests/bench_param_sweep.rs:71-72)."""
    i = np.arange(cfg.seq + 1, dtype=np.int64)
    s = ((i * 31 + 7) % cfg.vocab).astype(np.uint32)
    return np.tile(s[:-1], batch).copy(), np.tile(s[1:], batch).copy()


# ------------------------------------------------------------ model API
class Oracle:
    """Model-level oracle over `batch` sequences (reference channel-first math)."""

    def __init__(self, cfg: ModelConfig, batch: int = 1, threads: int | None = None):
        self.cfg = cfg
        self.c_cfg = cfg.to_c()
        self.L = lib(threads)
        self.batch = batch
        self.ws = self.L.or_ws_create(ctypes.byref(self.c_cfg), batch)

    def __del__(self):
        try:
            if self.ws:
                self.L.or_ws_destroy(self.ws)
        except Exception:
            pass

    def rope_tables(self):
        S, hd = self.cfg.seq, self.cfg.hd
        cf, sf = np.empty((S, hd), np.float32), np.empty((S, hd), np.float32)
        cb, sb = np.empty((hd // 2, S), np.float32), np.empty((hd // 2, S), np.float32)
        self.L.or_rope_tables(self.ws, fp(cf), fp(sf), fp(cb), fp(sb))
        return cf, sf, cb, sb

    def forward(self, w: ModelTensors, tokens, targets, softcap=0.0, want_logits=False, want_token_losses=False):
        n = tokens.size // self.cfg.seq
        assert n <= self.batch
        loss = ctypes.c_float()
        logits = np.empty((n * self.cfg.seq, self.cfg.vocab), np.float32) if want_logits else None
        tl = np.empty(n * self.cfg.seq, np.float32) if want_token_losses else None
        wp = w.c_ptrs()
        rc = self.L.or_forward(ctypes.byref(self.c_cfg), ctypes.byref(wp), up(tokens), up(targets), n, softcap,
                               self.ws, ctypes.byref(loss), fp(logits) if logits is not None else None,
                               fp(tl) if tl is not None else None)
        if rc != 0:
            raise ValueError(f"oracle forward failed: {rc}")
        return loss.value, logits, tl

    def backward(self, w: ModelTensors, tokens, grads: ModelTensors, softcap=0.0, loss_scale=1.0):
        n = tokens.size // self.cfg.seq
        wp, gp = w.c_ptrs(), grads.c_ptrs()
        self.L.or_backward(ctypes.byref(self.c_cfg), ctypes.byref(wp), self.ws, up(tokens), n, softcap, loss_scale,
                           ctypes.byref(gp))

    def grad_norm(self, grads: ModelTensors) -> float:
        gp = grads.c_ptrs()
        return self.L.or_grad_norm(ctypes.byref(self.c_cfg), ctypes.byref(gp))

    def update_weights(self, w, grads, opt: ModelOptState, t, lr, tc: OrTrainConfig, grad_scale):
        wp, gp, mp, vp = w.c_ptrs(), grads.c_ptrs(), opt.m.c_ptrs(), opt.v.c_ptrs()
        self.L.or_update_weights(ctypes.byref(self.c_cfg), ctypes.byref(wp), ctypes.byref(gp), ctypes.byref(mp),
                                 ctypes.byref(vp), t, lr, ctypes.byref(tc), grad_scale)

    def train_step(self, w, grads, opt: ModelOptState, tokens, targets, step, tc: OrTrainConfig):
        n = tokens.size // self.cfg.seq
        wp, gp, mp, vp = w.c_ptrs(), grads.c_ptrs(), opt.m.c_ptrs(), opt.v.c_ptrs()
        raw = ctypes.c_float()
        loss = self.L.or_train_step_batch(ctypes.byref(self.c_cfg), ctypes.byref(wp), ctypes.byref(gp),
                                          ctypes.byref(mp), ctypes.byref(vp), up(tokens), up(targets), n, step,
                                          ctypes.byref(tc), self.ws, ctypes.byref(raw))
        return loss, raw.value


    # ---- single layer (layer::forward / layer::backward / training::train_step), x in [D][S]
    def layer_forward(self, lw: LayerTensors, x: np.ndarray) -> np.ndarray:
        y = np.empty_like(x)
        wp = lw.c_ptrs()
        self.L.or_layer_forward(ctypes.byref(self.c_cfg), self.ws, ctypes.byref(wp), fp(x), fp(y))
        return y

    def layer_backward(self, lw: LayerTensors, dy: np.ndarray, g: LayerTensors) -> np.ndarray:
        dx = np.empty_like(dy)
        wp, gp = lw.c_ptrs(), g.c_ptrs()
        self.L.or_layer_backward(ctypes.byref(self.c_cfg), self.ws, ctypes.byref(wp), fp(dy), ctypes.byref(gp), fp(dx))
        return dx

    def layer_train_step(self, lw: LayerTensors, g: LayerTensors, m: LayerTensors, v: LayerTensors,
                         x: np.ndarray, t: int, lr: float, beta1: float = 0.9, beta2: float = 0.999,
                         eps: float = 1e-8, weight_decay: float = 0.01) -> float:
        ptrs = [a.c_ptrs() for a in (lw, g, m, v)]
        return self.L.or_layer_train_step(ctypes.byref(self.c_cfg), self.ws, *[ctypes.byref(p) for p in ptrs], fp(x),
                                          t, lr, beta1, beta2, eps, weight_decay)


def learning_rate(step: int, tc: OrTrainConfig) -> float:
    return lib().or_learning_rate(step, ctypes.byref(tc))
