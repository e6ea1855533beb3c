"""Engine API over librustane_cuda.so — the host-side mirror of the reference
engine crate's model API (crates/engine/src/full_model.rs, layer.rs,
training.rs), with the heavy work on a B200 through the C ABI.

Names and argument meaning follow the reference:

    kernels = CompiledKernels.compile(cfg)                 # layer.rs:237-275
    loss = full_model.forward(cfg, kernels, weights, tokens, targets, softcap)
    full_model.backward(cfg, kernels, weights, tokens, softcap, loss_scale, grads)
    full_model.update_weights(cfg, kernels, weights, grads, opt, t, lr, tc, grad_scale)
    loss = full_model.train_step(cfg, kernels, weights, grads, opt, data, step, tc)

Weights, gradients and Adam moments live on the device; the host containers
(rustane_b200.tensors) are synchronised explicitly: a `ModelWeights` passed to
forward() is uploaded when it is not the object last uploaded (or when
`weights.dirty` is set), and `grads` / `opt` arguments, when given, are
filled from the device after the call, so the calling code reads like the
reference's.  Errors raise RustaneError (the reference panics).
"""
from __future__ import annotations

import ctypes
from dataclasses import asdict, dataclass

import numpy as np

from . import _lib
from ._lib import RtTimings, RtTrainConfig, RustaneError, check, lib
from .model import ModelConfig
from .tensors import ModelOptState, ModelTensors


@dataclass
class TrainConfig:
    """TrainConfig::default (crates/engine/src/full_model.rs:51-70)."""
    max_lr: float = 3e-4
    min_lr_frac: float = 0.1
    warmup_steps: int = 100
    total_steps: int = 10000
    beta1: float = 0.9
    beta2: float = 0.95
    eps: float = 1e-8
    weight_decay: float = 0.1
    matrix_lr_scale: float = 0.05
    embed_lr_scale: float = 5.0
    loss_scale: float = 256.0
    accum_steps: int = 10
    grad_clip: float = 1.0
    softcap: float = 0.0

    def to_c(self) -> RtTrainConfig:
        return RtTrainConfig(**asdict(self))


def _u32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint32)
    return a


def _uptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))


def _fptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class CompiledKernels:
    """Holder of one rt_ctx (device arenas + stream) for a model config.

    Replaces CompiledKernels::compile (layer.rs:237-275) and the forward /
    backward workspaces (full_model.rs:123-185)."""

    def __init__(self, cfg: ModelConfig, handle: int, max_batch: int, forward_only: bool):
        self.cfg = cfg
        self._h = ctypes.c_void_p(handle)
        self.max_batch = max_batch
        self.forward_only = forward_only
        self._uploaded = None

    @classmethod
    def compile(cls, cfg: ModelConfig, max_batch: int = 1, device: int = 0,
                forward_only: bool = False) -> "CompiledKernels":
        h = ctypes.c_void_p()
        c_cfg = cfg.to_c()
        flags = _lib.RT_CTX_FORWARD_ONLY if forward_only else _lib.RT_CTX_TRAIN
        rc = lib().rt_ctx_create(ctypes.byref(c_cfg), device, max_batch, flags, ctypes.byref(h))
        if rc != _lib.RT_OK:
            raise RustaneError(rc, lib().rt_last_error(None).decode(errors="replace"))
        return cls(cfg, h.value, max_batch, forward_only)

    # ------------------------------------------------------------- lifecycle
    @property
    def handle(self):
        if self._h is None or not self._h.value:
            raise RuntimeError("CompiledKernels is closed")
        return self._h

    def close(self):
        if self._h is not None and self._h.value:
            lib().rt_ctx_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int):
        if rc != _lib.RT_OK:
            raise RustaneError(rc, lib().rt_last_error(self._h).decode(errors="replace"))

    def device_bytes(self) -> int:
        n = ctypes.c_int64()
        self._check(lib().rt_ctx_device_bytes(self.handle, ctypes.byref(n)))
        return n.value

    # --------------------------------------------------------- host <-> device
    def upload_weights(self, w: ModelTensors) -> None:
        p = w.c_ptrs()
        self._check(lib().rt_weights_upload(self.handle, ctypes.byref(p)))
        self._uploaded = w
        w.dirty = False

    def sync_weights(self, w: ModelTensors | None) -> None:
        if w is None:
            return
        if w is not self._uploaded or getattr(w, "dirty", False):
            self.upload_weights(w)

    def download_weights(self, w: ModelTensors | None = None) -> ModelTensors:
        w = w if w is not None else ModelTensors.zeros(self.cfg)
        p = w.c_ptrs()
        self._check(lib().rt_weights_download(self.handle, ctypes.byref(p)))
        return w

    def download_grads(self, g: ModelTensors | None = None) -> ModelTensors:
        g = g if g is not None else ModelTensors.zeros(self.cfg)
        p = g.c_ptrs()
        self._check(lib().rt_grads_download(self.handle, ctypes.byref(p)))
        return g

    def upload_grads(self, g: ModelTensors) -> None:
        p = g.c_ptrs()
        self._check(lib().rt_grads_upload(self.handle, ctypes.byref(p)))

    def download_opt(self, opt: ModelOptState | None = None) -> ModelOptState:
        opt = opt if opt is not None else ModelOptState.zeros(self.cfg)
        pm, pv = opt.m.c_ptrs(), opt.v.c_ptrs()
        self._check(lib().rt_opt_download(self.handle, ctypes.byref(pm), ctypes.byref(pv)))
        return opt

    def upload_opt(self, opt: ModelOptState) -> None:
        pm, pv = opt.m.c_ptrs(), opt.v.c_ptrs()
        self._check(lib().rt_opt_upload(self.handle, ctypes.byref(pm), ctypes.byref(pv)))

    def init_normal(self, seed: int = 1234, std: float = 0.02) -> None:
        self._check(lib().rt_weights_init_normal(self.handle, seed, std))
        self._uploaded = None

    # -------------------------------------------------------------- compute
    def forward(self, tokens, targets, softcap: float = 0.0, per_token: bool = False):
        tok, tgt = _u32(tokens), _u32(targets)
        batch = tok.size // self.cfg.seq
        if tok.size != batch * self.cfg.seq or tgt.size != tok.size:
            raise ValueError("tokens/targets must hold batch * seq ids")
        loss = ctypes.c_float()
        ptl = np.empty(tok.size, np.float32) if per_token else None
        self._check(lib().rt_forward(self.handle, _uptr(tok), _uptr(tgt), batch, softcap, ctypes.byref(loss),
                                     _fptr(ptl)))
        self._last_batch = batch
        return (loss.value, ptl) if per_token else loss.value

    def logits(self) -> np.ndarray:
        n = self._last_rows()
        out = np.empty((n, self.cfg.vocab), np.float32)
        self._check(lib().rt_logits_download(self.handle, _fptr(out)))
        return out

    def _last_rows(self) -> int:
        # the context keeps the batch of the last forward; rt_logits_download sizes by it
        return self._last_batch * self.cfg.seq

    def backward(self, softcap: float = 0.0, loss_scale: float = 1.0) -> None:
        self._check(lib().rt_backward(self.handle, softcap, loss_scale))

    def grads_zero(self) -> None:
        self._check(lib().rt_grads_zero(self.handle))

    def grad_norm(self) -> float:
        n = ctypes.c_float()
        self._check(lib().rt_grad_norm(self.handle, ctypes.byref(n)))
        return n.value

    def last_grad_norm(self) -> float:
        """The raw gradient norm the last train step computed on the device (no recompute, no gather)."""
        n = ctypes.c_float()
        self._check(lib().rt_last_grad_norm(self.handle, ctypes.byref(n)))
        return n.value

    def clip_grads(self, max_norm: float) -> None:
        self._check(lib().rt_clip_grads(self.handle, max_norm))

    def update_weights(self, t: int, lr: float, tc: TrainConfig, grad_scale: float) -> None:
        c_tc = tc.to_c()
        self._check(lib().rt_update_weights(self.handle, t, lr, ctypes.byref(c_tc), grad_scale))

    def train_step(self, tokens, targets, step: int, tc: TrainConfig) -> float:
        tok, tgt = _u32(tokens), _u32(targets)
        batch = tok.size // self.cfg.seq
        loss = ctypes.c_float()
        c_tc = tc.to_c()
        self._check(lib().rt_train_step(self.handle, _uptr(tok), _uptr(tgt), batch, step, ctypes.byref(c_tc),
                                        ctypes.byref(loss)))
        self._last_batch = batch
        return loss.value

    # -------------------------------------------------------- single layer
    # layer::forward / layer::backward / training::train_step on layer `layer` of
    # the uploaded weights; x, dy, y, dx per sequence in the reference's
    # channel-first [dim][seq] layout.
    def layer_forward(self, layer: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        batch = x.size // (self.cfg.dim * self.cfg.seq)
        y = np.empty_like(x)
        self._check(lib().rt_layer_forward(self.handle, layer, _fptr(x), batch, _fptr(y)))
        return y

    def layer_backward(self, layer: int, dy: np.ndarray) -> np.ndarray:
        dy = np.ascontiguousarray(dy, np.float32)
        dx = np.empty_like(dy)
        self._check(lib().rt_layer_backward(self.handle, layer, _fptr(dy), _fptr(dx)))
        return dx

    def layer_train_step(self, layer: int, x: np.ndarray, t: int, lr: float, beta1: float = 0.9,
                         beta2: float = 0.999, eps: float = 1e-8, weight_decay: float = 0.01) -> float:
        """training::train_step (training.rs:61-97); AdamConfig defaults of cpu/adam.rs:21-29."""
        x = np.ascontiguousarray(x, np.float32)
        batch = x.size // (self.cfg.dim * self.cfg.seq)
        ac = _lib.RtAdamConfig(lr, beta1, beta2, eps, weight_decay)
        loss = ctypes.c_float()
        self._check(lib().rt_layer_train_step(self.handle, layer, _fptr(x), batch, t, ctypes.byref(ac),
                                              ctypes.byref(loss)))
        return loss.value

    # ---------------------------------------------------------- multi-GPU
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        rc = lib().rt_nccl_unique_id(buf)
        if rc != _lib.RT_OK:
            raise RustaneError(rc, "ncclGetUniqueId")
        return bytes(buf)

    def dist_init(self, world: int, rank: int, unique_id: bytes | None, mode: int = _lib.RT_DIST_DATA_PARALLEL,
                  timeout_ms: int = 60000) -> None:
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id) if unique_id is not None else None
        self._check(lib().rt_dist_init(self.handle, world, rank, buf, mode, timeout_ms))

    def dist_ranks(self) -> int:
        """Ranks of this context's NCCL communicator (ncclCommCount); 1 without one."""
        n = ctypes.c_int()
        self._check(lib().rt_dist_ranks(self.handle, ctypes.byref(n)))
        return n.value

    def grad_allreduce(self) -> None:
        self._check(lib().rt_grad_allreduce(self.handle))

    # -------------------------------------------------------- diagnostics
    def profile(self, enable: bool) -> None:
        self._check(lib().rt_profile(self.handle, int(enable)))

    def timings(self) -> dict:
        t = RtTimings()
        self._check(lib().rt_get_timings(self.handle, ctypes.byref(t)))
        return {f: getattr(t, f) for f, _ in RtTimings._fields_}

    _last_batch = 1


# ------------------------------------------------------------------ full_model
def learning_rate(step: int, tc: TrainConfig) -> float:
    """full_model.rs:334-342."""
    c_tc = tc.to_c()
    return lib().rt_learning_rate(step, ctypes.byref(c_tc))


def tp_shard(heads: int, hidden: int, world: int, rank: int) -> tuple[int, int, int, int]:
    """The tensor-parallel partition of the library (rt_tp_shard): this rank's
    (head0, heads_loc, hid0, hid_loc)."""
    v = [ctypes.c_int() for _ in range(4)]
    check(lib().rt_tp_shard(heads, hidden, world, rank, *[ctypes.byref(x) for x in v]))
    return tuple(x.value for x in v)


def lcg_random_vec(n: int, scale: float) -> np.ndarray:
    """random_vec (layer.rs:404-413): the reference's deterministic init stream."""
    out = np.empty(n, np.float32)
    check(lib().rt_lcg_fill(_fptr(out), n, scale))
    return out


def random_weights(cfg: ModelConfig) -> ModelTensors:
    """ModelWeights::random (full_model.rs:84-90, layer.rs:358-373)."""
    t = ModelTensors.zeros(cfg)
    D, H = cfg.dim, cfg.hidden
    sq = np.float32(1.0) / np.sqrt(np.float32(D))
    sf = np.float32(1.0) / np.sqrt(np.float32(H))
    wq = lcg_random_vec(D * cfg.q_dim, float(sq))
    wk = wq if cfg.kv_dim == cfg.q_dim else lcg_random_vec(D * cfg.kv_dim, float(sq))
    w1 = lcg_random_vec(D * H, float(sf))
    for L in t.layers:
        L.wq[...] = wq.reshape(L.wq.shape)
        L.wk[...] = wk.reshape(L.wk.shape)
        L.wv[...] = wk.reshape(L.wv.shape)
        L.w1[...] = w1.reshape(L.w1.shape)
        L.w3[...] = w1.reshape(L.w3.shape)
        L.gamma1[...] = 1.0
        L.gamma2[...] = 1.0
    t.embed[...] = lcg_random_vec(cfg.vocab * D, 0.005).reshape(t.embed.shape)
    t.gamma_final[...] = 1.0
    return t


def forward(cfg: ModelConfig, kernels: CompiledKernels, weights: ModelTensors | None, tokens, targets,
            softcap: float = 0.0) -> float:
    """full_model::forward / forward_ws (full_model.rs:187-247, 345-414): mean loss."""
    kernels.sync_weights(weights)
    loss = kernels.forward(tokens, targets, softcap)
    kernels._last_batch = np.asarray(tokens).size // cfg.seq
    return loss


forward_ws = forward


def forward_losses(cfg: ModelConfig, kernels: CompiledKernels, weights: ModelTensors | None, tokens, targets,
                   softcap: float = 0.0) -> np.ndarray:
    """full_model::forward_losses (full_model.rs:717-767): per-token CE."""
    kernels.sync_weights(weights)
    _, ptl = kernels.forward(tokens, targets, softcap, per_token=True)
    kernels._last_batch = np.asarray(tokens).size // cfg.seq
    return ptl


def backward(cfg: ModelConfig, kernels: CompiledKernels, weights: ModelTensors | None, tokens, softcap: float,
             loss_scale: float, grads: ModelTensors | None = None) -> None:
    """full_model::backward / backward_ws (full_model.rs:250-331, 415-485).
    Gradients accumulate on the device; `grads`, when given, receives a copy."""
    kernels.backward(softcap, loss_scale)
    if grads is not None:
        kernels.download_grads(grads)


backward_ws = backward


def grad_norm(kernels: CompiledKernels) -> float:
    """full_model.rs:598-624."""
    return kernels.grad_norm()


def clip_grads(kernels: CompiledKernels, max_norm: float) -> None:
    """full_model.rs:627-645."""
    kernels.clip_grads(max_norm)


def update_weights(cfg: ModelConfig, kernels: CompiledKernels, weights: ModelTensors | None,
                   grads: ModelTensors | None, opt: ModelOptState | None, t: int, lr: float, tc: TrainConfig,
                   grad_scale: float) -> None:
    """full_model::update_weights (full_model.rs:490-593).  Host containers, when
    given, are refreshed from the device afterwards."""
    kernels.update_weights(t, lr, tc, grad_scale)
    if weights is not None:
        kernels.download_weights(weights)
        kernels._uploaded = weights
        weights.dirty = False
    if opt is not None:
        kernels.download_opt(opt)


def train_positions(step: int, accum_steps: int, n_data: int, seq: int) -> list[int]:
    """Microbatch positions of full_model::train_step (full_model.rs:678-682)."""
    max_pos = n_data - seq - 1
    return [(step * 7919 + micro * 104729) % max_pos for micro in range(accum_steps)]


def train_step(cfg: ModelConfig, kernels: CompiledKernels, weights: ModelTensors | None, grads, opt, data,
               step: int, tc: TrainConfig) -> float:
    """full_model::train_step (full_model.rs:661-714) on a u16 token stream:
    accum_steps microbatches at the reference's LCG positions, processed as one
    batch (gradients summed, loss averaged), clip, lr schedule, AdamW(step + 1)."""
    data = np.asarray(data)
    pos = train_positions(step, tc.accum_steps, data.size, cfg.seq)
    tok = np.concatenate([data[p:p + cfg.seq] for p in pos]).astype(np.uint32)
    tgt = np.concatenate([data[p + 1:p + cfg.seq + 1] for p in pos]).astype(np.uint32)
    kernels.sync_weights(weights)
    loss = kernels.train_step(tok, tgt, step, tc)
    if weights is not None:
        kernels.download_weights(weights)
        kernels._uploaded = weights
        weights.dirty = False
    if grads is not None:
        kernels.download_grads(grads)
    if opt is not None:
        kernels.download_opt(opt)
    return loss
