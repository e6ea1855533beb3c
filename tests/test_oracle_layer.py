"""Single-layer path of the oracle (layer::forward / layer::backward /
training::train_step, training.rs:61-97), pinned to the reference's own
Phase-3 test (tests/phase3_training.rs:10-52): GPT-Karpathy shapes, the
reference layer init, AdamConfig lr 1e-4 / wd 0, the input pattern
((i*7 + 13) % 200) * 0.01 - 1, loss decreasing over 10 steps."""
import numpy as np

import pyoracle as po
from rustane_b200.model import ModelConfig
from rustane_b200.tensors import LayerTensors


def _phase3_input(cfg):
    n = cfg.dim * cfg.seq
    i = np.arange(n, dtype=np.int64)
    return (((i * 7 + 13) % 200).astype(np.float32) * np.float32(0.01) - np.float32(1.0)).astype(np.float32)


def test_zero_init_layer_is_identity():
    # Wo = W2 = 0 (DeepNet init, layer.rs:358-373): both residual branches vanish
    cfg = ModelConfig.gpt_karpathy().with_(seq=128)
    lw = po.reference_init(cfg).layers[0].copy()
    x = _phase3_input(cfg)
    y = po.Oracle(cfg, 1).layer_forward(lw, x)
    assert np.array_equal(y, x)


def test_single_layer_loss_decreases():
    cfg = ModelConfig.gpt_karpathy()
    lw = po.reference_init(cfg).layers[0].copy()
    g, m, v = LayerTensors.zeros(cfg), LayerTensors.zeros(cfg), LayerTensors.zeros(cfg)
    x = _phase3_input(cfg)
    o = po.Oracle(cfg, 1)
    losses = [o.layer_train_step(lw, g, m, v, x, t, lr=1e-4, weight_decay=0.0) for t in range(1, 11)]
    # first step: the layer is the identity, so the loss is mean(x^2); the reference sums
    # 393216 squares sequentially in f32, which rounds at the 1e-4 relative level
    assert abs(losses[0] / float(np.mean(x.astype(np.float64) ** 2)) - 1.0) < 3e-4
    assert losses[-1] < losses[0]
    # only Wo and W2 move on step 1 (their inputs are the only non-zero paths); all nine move by step 10
    assert np.abs(lw.wo).max() > 0 and np.abs(lw.w2).max() > 0
