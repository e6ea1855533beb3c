"""Finite-difference check of the oracle's full-model backward (no GPU).

The reference pins its backward only loosely (loss decreases, non-zero grads);
the oracle's restatement of backward_into (crates/engine/src/layer.rs:1606-1858)
and backward_ws (full_model.rs:250-331) is checked here against central
differences of its own forward, for the largest-gradient entries of every
tensor, on a small random model where every path (attention, FFN, norms,
tied embedding) carries gradient.
"""
import numpy as np
import pytest

import pyoracle as po
from rustane_b200.model import ModelConfig
from rustane_b200.tensors import ModelTensors


@pytest.mark.parametrize("softcap", [0.0, 5.0])
def test_full_model_gradcheck(softcap):
    cfg = ModelConfig.custom(128, 256, 1, 2, seq=32, vocab=96)
    w = ModelTensors.normal(cfg, seed=11, std=0.08)
    rng = np.random.default_rng(4)
    for L in w.layers:
        L.gamma1[...] = 1 + 0.1 * rng.standard_normal(cfg.dim).astype(np.float32)
        L.gamma2[...] = 1 + 0.1 * rng.standard_normal(cfg.dim).astype(np.float32)
    tok = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    o = po.Oracle(cfg, 2)
    o.forward(w, tok, tgt, softcap=softcap)
    g = ModelTensors.zeros(cfg)
    o.backward(w, tok, g, softcap=softcap, loss_scale=1.0)

    def loss_of():
        return o.forward(w, tok, tgt, softcap=softcap)[0]

    # backward sums the per-sequence gradients of loss_b = CE_b / seq; the forward
    # returns their mean over the 2 sequences, so d(mean)/dw = grad / 2.
    checked = 0
    for (name, wa), (_, ga) in zip(w.tensors(), g.tensors()):
        flat_w, flat_g = wa.reshape(-1), ga.reshape(-1)
        for idx in np.argsort(-np.abs(flat_g))[:2]:
            if abs(flat_g[idx]) < 1e-4:
                continue
            eps = np.float32(2e-2 * max(abs(flat_w[idx]), 0.05))
            old = flat_w[idx]
            flat_w[idx] = old + eps
            lp = loss_of()
            flat_w[idx] = old - eps
            lm = loss_of()
            flat_w[idx] = old
            num = (lp - lm) / (2 * float(eps))
            ana = float(flat_g[idx]) / 2
            assert abs(num - ana) <= 0.05 * abs(ana) + 2e-4, (name, idx, num, ana)
            checked += 1
    assert checked >= 15
