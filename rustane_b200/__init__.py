"""rustane_b200 — B200-native (sm_100a) engine for rustane's language-model step.

The compute runs in librustane_cuda.so (include/rustane_cuda.h); this package
is the host-side mirror of the reference engine crate's API:

    from rustane_b200 import ModelConfig, CompiledKernels, TrainConfig, full_model
    kernels = CompiledKernels.compile(cfg, max_batch=8)
    loss = full_model.forward(cfg, kernels, weights, tokens, targets, 0.0)
"""
from . import engine as full_model
from ._lib import RustaneError
from .engine import CompiledKernels, TrainConfig, learning_rate, random_weights
from .model import ModelConfig
from .tensors import ModelGrads, ModelOptState, ModelTensors, ModelWeights

__all__ = ["ModelConfig", "ModelWeights", "ModelGrads", "ModelOptState", "ModelTensors", "TrainConfig",
           "CompiledKernels", "full_model", "learning_rate", "random_weights", "RustaneError"]
