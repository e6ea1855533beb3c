"""Model configuration (mirror of crates/engine/src/model.rs:5-152).

`ModelConfig` carries the same fields as the reference struct and is passed to
the C ABI as `rt_model_config`.  Presets reproduce the reference's constructors
plus the five configurations the B200 benchmarks are quoted on.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace


class RtModelConfig(ctypes.Structure):
    """C layout of rt_model_config (include/rustane_cuda.h)."""
    _fields_ = [(n, ctypes.c_int32) for n in
                ("dim", "hidden", "heads", "kv_heads", "hd", "seq", "nlayers", "vocab", "q_dim", "kv_dim",
                 "gqa_ratio")]


@dataclass(frozen=True)
class ModelConfig:
    dim: int
    hidden: int
    heads: int
    kv_heads: int
    hd: int
    seq: int
    nlayers: int
    vocab: int
    q_dim: int
    kv_dim: int
    gqa_ratio: int

    # ---- reference presets (model.rs:19-151)
    @staticmethod
    def custom(dim: int, hidden: int, heads: int, nlayers: int, seq: int = 512, vocab: int = 8192,
               hd: int = 128) -> "ModelConfig":
        """MHA config with head_dim 128 (tests/bench_param_sweep.rs:18-29)."""
        return ModelConfig(dim=dim, hidden=hidden, heads=heads, kv_heads=heads, hd=hd, seq=seq, nlayers=nlayers,
                           vocab=vocab, q_dim=heads * hd, kv_dim=heads * hd, gqa_ratio=1)

    @staticmethod
    def gpt_karpathy() -> "ModelConfig":  # model.rs:21-35
        return ModelConfig.custom(768, 2048, 6, 6)

    @staticmethod
    def gpt_1024() -> "ModelConfig":  # model.rs:38-52
        return ModelConfig.custom(1024, 2816, 8, 8)

    @staticmethod
    def target_600m() -> "ModelConfig":  # model.rs:56-70
        return ModelConfig.custom(1536, 4096, 12, 20)

    @staticmethod
    def target_800m() -> "ModelConfig":  # model.rs:74-88
        return ModelConfig.custom(1792, 4864, 14, 24)

    @staticmethod
    def target_1b() -> "ModelConfig":  # model.rs:92-106
        return ModelConfig.custom(2048, 5632, 16, 28)

    @staticmethod
    def target_1_5b() -> "ModelConfig":  # model.rs:118-132
        return ModelConfig.custom(2304, 6144, 18, 32)

    @staticmethod
    def mha_28l() -> "ModelConfig":  # model.rs:137-151
        return ModelConfig.custom(1024, 3072, 8, 28, seq=256)

    # ---- benchmark configurations (BASELINE configs[0..4])
    @staticmethod
    def tiny() -> "ModelConfig":
        return ModelConfig.gpt_karpathy()

    @staticmethod
    def c600m() -> "ModelConfig":
        return ModelConfig.target_600m()

    @staticmethod
    def c5b() -> "ModelConfig":
        return ModelConfig.custom(2560, 6912, 20, 60)

    @staticmethod
    def c7b() -> "ModelConfig":
        return ModelConfig.custom(4096, 11008, 32, 32)

    @staticmethod
    def c30b() -> "ModelConfig":
        return ModelConfig.custom(6656, 17920, 52, 60)

    def with_(self, **kw) -> "ModelConfig":
        return replace(self, **kw)

    def param_count(self) -> int:
        """model.rs:109-114."""
        per_layer = 4 * self.dim * self.dim + 3 * self.dim * self.hidden
        return self.nlayers * per_layer + self.vocab * self.dim + self.dim * (2 * self.nlayers + 1)

    def flops_per_token_fwd(self) -> float:
        """Algorithmic forward FLOPs per token: projections, FFN, logits, causal attention."""
        L, D, H, V, S = self.nlayers, self.dim, self.hidden, self.vocab, self.seq
        return 2.0 * L * (4 * D * D + 3 * D * H) + 2.0 * D * V + 2.0 * L * S * D

    def to_c(self) -> RtModelConfig:
        return RtModelConfig(self.dim, self.hidden, self.heads, self.kv_heads, self.hd, self.seq, self.nlayers,
                             self.vocab, self.q_dim, self.kv_dim, self.gqa_ratio)
