"""Host-side parameter containers in the reference layouts.

Mirrors LayerWeights / LayerGrads (crates/engine/src/layer.rs:16-39),
ModelWeights / ModelGrads / ModelOptState (crates/engine/src/full_model.rs:13-31,
84-121) and LayerOptState (crates/engine/src/training.rs:11-37).  Arrays are
C-contiguous float32 numpy arrays: wq/wk/wv [dim, q_dim|kv_dim], wo [q_dim, dim],
w1/w3/w2 [dim, hidden], gamma1/gamma2 [dim], embed [vocab, dim],
gamma_final [dim].  Gradients and Adam moments use the same container with the
same field names (the reference prefixes them with d / m_ / v_).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from .model import ModelConfig

LAYER_FIELDS = ("wq", "wk", "wv", "wo", "w1", "w3", "w2", "gamma1", "gamma2")
MATRIX_FIELDS = ("wq", "wk", "wv", "wo", "w1", "w3", "w2")


def layer_shapes(cfg: ModelConfig) -> dict[str, tuple[int, ...]]:
    D, Q, KV, H = cfg.dim, cfg.q_dim, cfg.kv_dim, cfg.hidden
    return {"wq": (D, Q), "wk": (D, KV), "wv": (D, KV), "wo": (Q, D), "w1": (D, H), "w3": (D, H), "w2": (D, H),
            "gamma1": (D,), "gamma2": (D,)}


class RtLayerPtrs(ctypes.Structure):
    _fields_ = [(n, ctypes.POINTER(ctypes.c_float)) for n in LAYER_FIELDS]


class RtModelPtrs(ctypes.Structure):
    _fields_ = [("embed", ctypes.POINTER(ctypes.c_float)), ("gamma_final", ctypes.POINTER(ctypes.c_float)),
                ("layers", ctypes.POINTER(RtLayerPtrs))]


def _fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


@dataclass
class LayerTensors:
    wq: np.ndarray
    wk: np.ndarray
    wv: np.ndarray
    wo: np.ndarray
    w1: np.ndarray
    w3: np.ndarray
    w2: np.ndarray
    gamma1: np.ndarray
    gamma2: np.ndarray

    def arrays(self):
        return [getattr(self, f) for f in LAYER_FIELDS]

    @classmethod
    def zeros(cls, cfg: ModelConfig) -> "LayerTensors":
        return cls(**{n: np.zeros(shp, np.float32) for n, shp in layer_shapes(cfg).items()})

    def copy(self) -> "LayerTensors":
        return LayerTensors(*[a.copy() for a in self.arrays()])

    def c_ptrs(self) -> RtLayerPtrs:
        return RtLayerPtrs(*[_fptr(a) for a in self.arrays()])


@dataclass
class ModelTensors:
    cfg: ModelConfig
    embed: np.ndarray
    gamma_final: np.ndarray
    layers: list = field(default_factory=list)
    _c_layers: object = field(default=None, repr=False)

    # ------------------------------------------------------------ builders
    @classmethod
    def zeros(cls, cfg: ModelConfig) -> "ModelTensors":
        shapes = layer_shapes(cfg)
        layers = [LayerTensors(**{k: np.zeros(s, np.float32) for k, s in shapes.items()})
                  for _ in range(cfg.nlayers)]
        return cls(cfg, np.zeros((cfg.vocab, cfg.dim), np.float32), np.zeros(cfg.dim, np.float32), layers)

    @classmethod
    def normal(cls, cfg: ModelConfig, seed: int = 1234, std: float = 0.02) -> "ModelTensors":
        """Weights N(0, std) from a seed, gammas = 1 (the benchmark init)."""
        rng = np.random.default_rng(seed)
        t = cls.zeros(cfg)
        t.embed[...] = rng.normal(0.0, std, t.embed.shape).astype(np.float32)
        t.gamma_final[...] = 1.0
        for L in t.layers:
            for f in MATRIX_FIELDS:
                a = getattr(L, f)
                a[...] = rng.normal(0.0, std, a.shape).astype(np.float32)
            L.gamma1[...] = 1.0
            L.gamma2[...] = 1.0
        return t

    # ------------------------------------------------------------- helpers
    def tensors(self):
        """(name, array) in the reference's grad-norm / Adam order (full_model.rs:598-624)."""
        yield "embed", self.embed
        yield "gamma_final", self.gamma_final
        for i, L in enumerate(self.layers):
            for f in LAYER_FIELDS:
                yield f"layers.{i}.{f}", getattr(L, f)

    def copy(self) -> "ModelTensors":
        out = ModelTensors.zeros(self.cfg)
        for (_, a), (_, b) in zip(out.tensors(), self.tensors()):
            a[...] = b
        return out

    def c_ptrs(self) -> RtModelPtrs:
        """ctypes view (rt_model_ptrs / the oracle's OrModel); keeps arrays referenced."""
        arr = (RtLayerPtrs * max(1, len(self.layers)))()
        for i, L in enumerate(self.layers):
            arr[i] = RtLayerPtrs(*[_fptr(a) for a in L.arrays()])
        self._c_layers = arr
        return RtModelPtrs(_fptr(self.embed), _fptr(self.gamma_final), arr)


ModelWeights = ModelTensors
ModelGrads = ModelTensors


@dataclass
class ModelOptState:
    """Adam first/second moments (full_model.rs:26-31)."""
    m: ModelTensors
    v: ModelTensors

    @classmethod
    def zeros(cls, cfg: ModelConfig) -> "ModelOptState":
        return cls(ModelTensors.zeros(cfg), ModelTensors.zeros(cfg))
